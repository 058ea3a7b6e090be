"""GPU: the ViT attention block (the path's caller) against an fp32 torch
reference block with the same weights, where the attention is the oracle's
restatement of the reference harness (PyTorch SDPA + Python 2D RoPE)."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _rope_sdpa_fp32(q, k, v, cos, sin, has_cls):
    import torch.nn.functional as F
    N = q.shape[-2]
    off = 1 if has_cls else 0
    C = torch.ones(N, cos.shape[1], device=q.device)
    S = torch.zeros(N, cos.shape[1], device=q.device)
    C[off:], S[off:] = cos[: N - off], sin[: N - off]

    def rot(x):
        e, o = x[..., 0::2], x[..., 1::2]
        return torch.stack((e * C - o * S, o * C + e * S), dim=-1).flatten(-2)

    return F.scaled_dot_product_attention(rot(q), rot(k), v)


@pytest.mark.parametrize("dim,heads,side,has_cls", [(384, 6, 14, True), (256, 4, 8, False)])
def test_block_matches_fp32_reference(dim, heads, side, has_cls):
    from triton_fused_rope_flash_attn_b200.block import RopeAttention
    torch.manual_seed(0)
    blk = RopeAttention(dim, heads, H_img=side, has_cls=has_cls, device="cuda",
                        dtype=torch.bfloat16)
    N = side * side + (1 if has_cls else 0)
    x = torch.randn(3, N, dim, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    y = blk(x)
    gy = torch.randn_like(y)
    y.backward(gy)

    # fp32 reference with the same (bf16-valued) weights and input.
    W, b = blk.qkv.weight.float(), blk.qkv.bias.float()
    Wp, bp = blk.proj.weight.float(), blk.proj.bias.float()
    xr = x.detach().float().requires_grad_(True)
    D = dim // heads
    qkv = (xr @ W.t() + b).view(3, N, 3, heads, D).permute(2, 0, 3, 1, 4)
    o = _rope_sdpa_fp32(qkv[0], qkv[1], qkv[2], blk.rope.COSP, blk.rope.SINP, has_cls)
    yr = o.transpose(1, 2).reshape(3, N, dim) @ Wp.t() + bp
    yr.backward(gy.float())

    def rel(a, b):
        return float((a.float() - b).abs().max() / b.abs().max())

    assert rel(y.detach(), yr.detach()) < 2e-2
    assert rel(x.grad, xr.grad) < 3e-2


@pytest.mark.parametrize("dim,heads,side,has_cls", [(768, 12, 14, True), (384, 6, 7, False)])
def test_fused_qkv_rope_block_matches_unfused(dim, heads, side, has_cls):
    """RoPE in the QKV-projection epilogue (frsa_qkv_rope) + attention without
    rotation (rope=False), against the same block on the unfused path (same weights):
    output and the gradients of x, W_qkv and b_qkv."""
    from triton_fused_rope_flash_attn_b200.block import RopeAttention
    torch.manual_seed(1)
    ref = RopeAttention(dim, heads, H_img=side, has_cls=has_cls, device="cuda",
                        dtype=torch.bfloat16)
    fused = RopeAttention(dim, heads, H_img=side, has_cls=has_cls, device="cuda",
                          dtype=torch.bfloat16, fused_qkv=True)
    fused.load_state_dict(ref.state_dict())
    N = side * side + (1 if has_cls else 0)
    x0 = torch.randn(2, N, dim, device="cuda", dtype=torch.bfloat16)
    outs = []
    for blk in (ref, fused):
        x = x0.clone().requires_grad_(True)
        y = blk(x)
        y.backward(torch.ones_like(y))
        outs.append((y.detach().float(), x.grad.float(), blk.qkv.weight.grad.float(),
                     blk.qkv.bias.grad.float()))
    for a, b in zip(*outs):
        assert float((a - b).abs().max() / b.abs().max()) < 2e-2
