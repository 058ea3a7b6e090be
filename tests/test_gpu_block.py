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
