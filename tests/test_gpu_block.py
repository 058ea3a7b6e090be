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


@pytest.mark.parametrize("B,C,H,side,has_cls,dtype", [(2, 768, 12, 14, True, torch.bfloat16),
                                                      (1, 384, 6, 7, False, torch.float16)])
def test_qkv_rope_bwd_kernel_matches_torch(B, C, H, side, has_cls, dtype):
    """frsa_qkv_rope_bwd through the C ABI against its definition in fp32 torch:
    dqkv[b*N + n] = concat over q, k, v of the head-merged gradients, with R^T
    (the reference's pair rotation transposed) on the q and k parts."""
    from triton_fused_rope_flash_attn_b200 import CosSinTable, _lib
    N = side * side + (1 if has_cls else 0)
    D = C // H
    cs = CosSinTable(100.0, side, D, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(3)
    dq, dk, dv = (torch.randn(B, H, N, D, device="cuda", generator=g).to(dtype) for _ in range(3))
    dqkv = torch.empty(B * N, 3 * C, device="cuda", dtype=dtype)
    a = _lib.FrsaQkvBwdArgs()
    a.dq, a.dk, a.dv = dq.data_ptr(), dk.data_ptr(), dv.data_ptr()
    a.cosp, a.sinp, a.dqkv = cs.COSP.data_ptr(), cs.SINP.data_ptr(), dqkv.data_ptr()
    a.B, a.N, a.C, a.H, a.n_pos = B, N, C, H, cs.COSP.shape[0]
    a.has_cls, a.dtype = int(has_cls), (_lib.FRSA_DTYPE_BF16 if dtype == torch.bfloat16
                                        else _lib.FRSA_DTYPE_F16)
    assert _lib.load().frsa_qkv_rope_bwd(a, None) == 0
    torch.cuda.synchronize()
    off = 1 if has_cls else 0
    c = torch.ones(N, D // 2, device="cuda")
    s = torch.zeros(N, D // 2, device="cuda")
    c[off:], s[off:] = cs.COSP[: N - off], cs.SINP[: N - off]
    parts = []
    for t, rot in ((dq, True), (dk, True), (dv, False)):
        t = t.float()
        if rot:
            e, o = t[..., 0::2], t[..., 1::2]
            t = torch.stack((e * c + o * s, o * c - e * s), dim=-1).flatten(-2)
        parts.append(t.transpose(1, 2).reshape(B * N, C))
    ref = torch.cat(parts, dim=-1)
    err = (dqkv.float() - ref).abs().max().item()
    assert err <= 2 ** -7 * ref.abs().max().item(), err
