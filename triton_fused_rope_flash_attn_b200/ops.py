"""``torch.library`` registration of the fused 2D-RoPE attention.

The reference exposes the kernel only through a ``torch.autograd.Function``
(fa_rope_full .py:1011-1170), which ``torch.compile`` cannot trace into: a
compiled model graph-breaks around every attention call. Registering the
forward and backward as custom ops with fake (shape-only) implementations lets
``torch.compile`` keep the attention inside one graph, calling the same C ABI
as ``TritonAttention`` at run time.

Ops (namespace ``frsa``):

* ``frsa::attn_fwd(q, k, v, cosp, sinp, has_cls) -> (o, lse)``
* ``frsa::attn_bwd(q, k, v, o, lse, d_o, cosp, sinp, has_cls) -> (dq, dk, dv)``

``attn_fwd`` carries an autograd formula that calls ``attn_bwd``.
``sdpa_fa_rope_op`` is the differentiable entry with the reference's dtype
rule (compute in the autocast dtype when autocast is on, outputs in the input
dtype).
"""
from __future__ import annotations

import math
from typing import Tuple

import torch
from torch import Tensor

from .attention import (TritonAttention, _check_tables, _sdpa_comp_dtype,
                        fused_rope_attention_bwd, fused_rope_attention_fwd)


@torch.library.custom_op("frsa::attn_fwd", mutates_args=())
def attn_fwd(q: Tensor, k: Tensor, v: Tensor, cosp: Tensor, sinp: Tensor,
             has_cls: bool) -> Tuple[Tensor, Tensor]:
    """Forward: ``o`` (q's dtype) and the natural-log row LSE (float32 ``[B, H, N]``)."""
    return fused_rope_attention_fwd(q, k, v, cosp, sinp, has_cls)


@attn_fwd.register_fake
def _attn_fwd_fake(q, k, v, cosp, sinp, has_cls):
    B, H, N, _ = q.shape
    return (torch.empty(q.shape, dtype=q.dtype, device=q.device),
            torch.empty((B, H, N), dtype=torch.float32, device=q.device))


@torch.library.custom_op("frsa::attn_bwd", mutates_args=())
def attn_bwd(q: Tensor, k: Tensor, v: Tensor, o: Tensor, lse: Tensor, d_o: Tensor,
             cosp: Tensor, sinp: Tensor, has_cls: bool) -> Tuple[Tensor, Tensor, Tensor]:
    """Backward: ``(dq, dk, dv)`` in q's dtype."""
    return fused_rope_attention_bwd(q, k, v, o, lse, d_o, cosp, sinp, has_cls)


@attn_bwd.register_fake
def _attn_bwd_fake(q, k, v, o, lse, d_o, cosp, sinp, has_cls):
    return (torch.empty(q.shape, dtype=q.dtype, device=q.device),
            torch.empty(k.shape, dtype=k.dtype, device=k.device),
            torch.empty(v.shape, dtype=v.dtype, device=v.device))


def _setup_context(ctx, inputs, output):
    q, k, v, cosp, sinp, has_cls = inputs
    o, lse = output
    ctx.save_for_backward(q, k, v, o, lse, cosp, sinp)
    ctx.has_cls = has_cls
    ctx.mark_non_differentiable(lse)


def _backward(ctx, d_o, _d_lse):
    q, k, v, o, lse, cosp, sinp = ctx.saved_tensors
    dq, dk, dv = attn_bwd(q, k, v, o, lse, d_o.contiguous(), cosp, sinp, ctx.has_cls)
    return dq, dk, dv, None, None, None


attn_fwd.register_autograd(_backward, setup_context=_setup_context)


def sdpa_fa_rope_op(Q: Tensor, K: Tensor, V: Tensor, cos_sin, *, has_cls: bool = True) -> Tensor:
    """Differentiable fused 2D-RoPE SDPA through the registered ops.

    Same result and dtype rule as ``sdpa_triton_fa_rope`` (fa_rope_full
    .py:1169-1170); traceable by ``torch.compile`` without a graph break.
    """
    D = Q.shape[-1]
    assert (D % 4) == 0, "HEAD_DIM must be divisible by 4 (2D RoPE requires pairs)."
    comp = _sdpa_comp_dtype(Q)
    if comp == torch.float32 or Q.dtype == torch.float32:
        # float32 compute picks per-call power-of-two range factors from the
        # data, which a traced graph cannot hold, and float32 inputs under
        # 16-bit autocast go through the fused conversion kernels: both run
        # through the autograd.Function path (eager).
        return TritonAttention.apply(Q, K, V, cos_sin, math.isqrt(cos_sin.tables()[0].shape[0]),
                                     has_cls)
    COSP, SINP = cos_sin.tables()
    _check_tables(COSP, SINP, Q.shape[-2], D, has_cls, Q.device)
    q, k, v = (t.to(comp).contiguous() for t in (Q, K, V))
    o, _ = attn_fwd(q, k, v, COSP.contiguous(), SINP.contiguous(), has_cls)
    return o.to(Q.dtype)
