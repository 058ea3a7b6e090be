"""The QKV projection with the 2D RoPE fused into its epilogue.

``qkv_rope(x, weight, bias, cos_sin, num_heads, has_cls)`` computes what a ViT
attention block does before the attention (reference README:156-159: timm's
``qkv = Linear(x)``, head split, RoPE on q and k) in one sm_100a kernel
(``frsa_qkv_rope`` of the C ABI): a tcgen05 GEMM whose epilogue adds the bias,
rotates q and k by token position and writes q, k, v as ``[B, H, N, D]``.
The attention over these q, k then runs with ``rope=False`` (the C ABI's
FRSA_FLAG_NO_ROPE: the kernels rotate nothing), so the rotation leaves the
attention kernels. The backward is one kernel (``frsa_qkv_rope_bwd``) that
applies ``R^T`` to dq and dk and merges the heads back into the projection
output's gradient ``[B*N, 3C]``, then two GEMMs for dx and dW.
"""
from __future__ import annotations

import torch

from . import _lib


def supported(C: int, num_heads: int, dtype: torch.dtype) -> bool:
    """Shapes and dtypes the fused kernel handles (else use the unfused path)."""
    D = C // num_heads
    return (C % num_heads == 0 and C % 128 == 0 and D % 32 == 0 and D <= 128
            and dtype in (torch.bfloat16, torch.float16))


class QKVRope(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, cosp, sinp, num_heads: int, has_cls: bool):
        B, N, C = x.shape
        D = C // num_heads
        x2 = x.contiguous()
        w = weight.contiguous()
        b32 = (bias if bias is not None else torch.zeros(3 * C, device=x.device)).float().contiguous()
        q, k, v = (torch.empty(B, num_heads, N, D, device=x.device, dtype=x.dtype)
                   for _ in range(3))
        a = _lib.FrsaQkvArgs()
        a.x, a.w, a.bias = x2.data_ptr(), w.data_ptr(), b32.data_ptr()
        a.cosp, a.sinp = cosp.data_ptr(), sinp.data_ptr()
        a.q, a.k, a.v = q.data_ptr(), k.data_ptr(), v.data_ptr()
        a.B, a.N, a.C, a.H, a.n_pos = B, N, C, num_heads, cosp.shape[0]
        a.has_cls = int(bool(has_cls))
        a.dtype = _lib.FRSA_DTYPE_BF16 if x.dtype == torch.bfloat16 else _lib.FRSA_DTYPE_F16
        _lib.check(_lib.load().frsa_qkv_rope(a, torch.cuda.current_stream(x.device).cuda_stream),
                   "frsa_qkv_rope")
        ctx.save_for_backward(x2, w, cosp, sinp)
        ctx.has_bias = bias is not None
        ctx.meta = (num_heads, has_cls)
        return q, k, v

    @staticmethod
    def backward(ctx, dq, dk, dv):
        # One kernel (frsa_qkv_rope_bwd) turns dq, dk, dv into the gradient of
        # the projection output, dqkv [B*N, 3C] (R^T on the q and k parts);
        # the weight and input gradients are then two plain GEMMs.
        x, w, cosp, sinp = ctx.saved_tensors
        num_heads, has_cls = ctx.meta
        B, N, C = x.shape
        D = C // num_heads
        grads = []
        for g in (dq, dk, dv):
            g = torch.zeros(B, num_heads, N, D, device=x.device, dtype=x.dtype) if g is None \
                else g.to(x.dtype).contiguous()
            grads.append(g)
        dqkv = torch.empty(B * N, 3 * C, device=x.device, dtype=x.dtype)
        a = _lib.FrsaQkvBwdArgs()
        a.dq, a.dk, a.dv = (g.data_ptr() for g in grads)
        a.cosp, a.sinp = cosp.data_ptr(), sinp.data_ptr()
        a.dqkv = dqkv.data_ptr()
        a.B, a.N, a.C, a.H, a.n_pos = B, N, C, num_heads, cosp.shape[0]
        a.has_cls = int(bool(has_cls))
        a.dtype = _lib.FRSA_DTYPE_BF16 if x.dtype == torch.bfloat16 else _lib.FRSA_DTYPE_F16
        _lib.check(_lib.load().frsa_qkv_rope_bwd(
            a, torch.cuda.current_stream(x.device).cuda_stream), "frsa_qkv_rope_bwd")
        dx = (dqkv @ w).view(B, N, C)                          # [B, N, C]
        dw = dqkv.t() @ x.reshape(-1, C)                       # [3C, C]
        db = dqkv.float().sum(dim=0) if ctx.has_bias else None
        return dx, dw, db, None, None, None, None


def qkv_rope(x, weight, bias, cos_sin, num_heads: int, has_cls: bool = True):
    """``(q, k, v)`` as ``[B, H, N, D]``, q and k already rotated (see module doc)."""
    COSP, SINP = cos_sin.tables()
    return QKVRope.apply(x, weight, bias, COSP.contiguous(), SINP.contiguous(), num_heads,
                         has_cls)
