"""CPU restatement of the reference's fused 2D-RoPE attention (TEST INFRASTRUCTURE).

This module is the parity oracle. It is imported only by tests, by
``__graft_entry__.smoke()`` as the checker, and by ``bench.py``'s CPU-baseline
leg. It is never on the product path.

Reference being restated: ``fa_rope_full .py`` of v1kstrand/triton_fused_rope_flash_attn.

* Tables: ``build_axial_rope_pairs`` (fa_rope_full .py:10-63). Pair column
  ``k < D/4`` takes angle ``row * inv_freq[k]`` where ``row = lin // side``;
  pair column ``D/4 + k`` takes ``col * inv_freq[k]`` where ``col = lin % side``;
  ``inv_freq[k] = base ** (-k / (D/4))`` (fa_rope_full .py:35-61).
* Positions: token ``t`` uses table row ``t - has_cls``; the CLS token (t == 0
  when has_cls) is not rotated (fa_rope_full .py:177-179, 201-202, 249-251, 271-272).
* Rotation of pair (2p, 2p+1): ``e' = e*c - o*s``, ``o' = o*c + e*s``.
* Logits ``S = R(q) R(k)^T / sqrt(D)``, softmax, ``O = P V``, and the stored
  log-sum-exp ``M = max + ln(sum)`` (fa_rope_full .py:275-315, 1024).
* Backward: ``Delta = rowsum(dO * O)`` (fa_rope_full .py:352-357);
  ``dS = P (dO V^T - Delta)``; ``dQ^ = scale dS K^``, ``dK^ = scale dS^T Q^``,
  ``dV = P^T dO``; gradients are un-rotated with ``R^T``:
  ``de = de^ c + do^ s``, ``do = -de^ s + do^ c`` (fa_rope_full .py:620-662, 954-993).

The numpy functions compute in float64. ``attn_fwd_bwd_torch`` restates the
reference's described correctness harness ("PyTorch SDPA + Python RoPE",
README.md:123-136) with torch autograd and is the timed CPU baseline.
"""
from __future__ import annotations

import math

import numpy as np


def rope_tables_np(side: int, head_dim: int, base: float = 10000.0, dtype=np.float32):
    """Pairwise axial RoPE tables ``(cos, sin)`` of shape ``[side*side, head_dim//2]``.

    Follows fa_rope_full .py:10-63. The reference computes ``inv_freq`` and the
    angles in float32 (torch default dtype); ``dtype=np.float32`` mirrors that
    rounding so the result can be compared bitwise-or-ulp with the reference.
    """
    assert head_dim % 4 == 0, "need head_dim divisible by 4 for 2D axial RoPE"
    P = head_dim // 4
    k = np.arange(P, dtype=np.float64)
    expo = (-k / P).astype(dtype)
    inv_freq = np.power(dtype(base), expo).astype(dtype)       # fa_rope_full .py:35
    lin = np.arange(side * side)
    row = (lin // side).astype(dtype)                           # outer index, fa_rope_full .py:46-47
    col = (lin % side).astype(dtype)                            # inner index, fa_rope_full .py:50-51
    ang_r = (row[:, None] * inv_freq[None, :]).astype(dtype)
    ang_c = (col[:, None] * inv_freq[None, :]).astype(dtype)
    cos = np.concatenate([np.cos(ang_r), np.cos(ang_c)], axis=1).astype(dtype)
    sin = np.concatenate([np.sin(ang_r), np.sin(ang_c)], axis=1).astype(dtype)
    return np.ascontiguousarray(cos), np.ascontiguousarray(sin)


def _pos_tables(cos, sin, N: int, has_cls: bool):
    """Per-token (C, S) of shape [N, D/2]; CLS row gets the identity (1, 0)."""
    D2 = cos.shape[1]
    C = np.ones((N, D2), dtype=np.float64)
    S = np.zeros((N, D2), dtype=np.float64)
    off = 1 if has_cls else 0
    C[off:] = cos[: N - off]
    S[off:] = sin[: N - off]
    return C, S


def rotate_pairs_np(x, cos, sin, has_cls: bool):
    """Apply R to ``x[..., N, D]`` (fa_rope_full .py:201-202)."""
    x = np.asarray(x, dtype=np.float64)
    N = x.shape[-2]
    C, S = _pos_tables(cos, sin, N, has_cls)
    e, o = x[..., 0::2], x[..., 1::2]
    out = np.empty_like(x)
    out[..., 0::2] = e * C - o * S
    out[..., 1::2] = o * C + e * S
    return out


def unrotate_pairs_np(g, cos, sin, has_cls: bool):
    """Apply R^T to a gradient ``g[..., N, D]`` (fa_rope_full .py:653-662)."""
    g = np.asarray(g, dtype=np.float64)
    N = g.shape[-2]
    C, S = _pos_tables(cos, sin, N, has_cls)
    e, o = g[..., 0::2], g[..., 1::2]
    out = np.empty_like(g)
    out[..., 0::2] = e * C + o * S
    out[..., 1::2] = -e * S + o * C
    return out


def attn_fwd_np(q, k, v, cos, sin, has_cls: bool = True):
    """Forward: returns ``(O, M)`` with ``M = rowmax + ln(rowsum)`` (natural log)."""
    D = q.shape[-1]
    scale = 1.0 / math.sqrt(D)
    qr = rotate_pairs_np(q, cos, sin, has_cls)
    kr = rotate_pairs_np(k, cos, sin, has_cls)
    s = np.einsum("...id,...jd->...ij", qr, kr) * scale
    m = s.max(axis=-1, keepdims=True)
    p = np.exp(s - m)
    l = p.sum(axis=-1, keepdims=True)
    o = np.einsum("...ij,...jd->...id", p / l, np.asarray(v, dtype=np.float64))
    lse = (m + np.log(l))[..., 0]
    return o, lse


def attn_bwd_np(q, k, v, do, cos, sin, has_cls: bool = True):
    """Backward: returns ``(dQ, dK, dV)`` by the analytic formulas of the reference."""
    D = q.shape[-1]
    scale = 1.0 / math.sqrt(D)
    v = np.asarray(v, dtype=np.float64)
    do = np.asarray(do, dtype=np.float64)
    qr = rotate_pairs_np(q, cos, sin, has_cls)
    kr = rotate_pairs_np(k, cos, sin, has_cls)
    s = np.einsum("...id,...jd->...ij", qr, kr) * scale
    s = s - s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p = p / p.sum(axis=-1, keepdims=True)
    o = np.einsum("...ij,...jd->...id", p, v)
    delta = (do * o).sum(axis=-1, keepdims=True)
    dp = np.einsum("...id,...jd->...ij", do, v)
    ds = p * (dp - delta)
    dqr = np.einsum("...ij,...jd->...id", ds, kr) * scale
    dkr = np.einsum("...ij,...id->...jd", ds, qr) * scale
    dv = np.einsum("...ij,...id->...jd", p, do)
    return unrotate_pairs_np(dqr, cos, sin, has_cls), unrotate_pairs_np(dkr, cos, sin, has_cls), dv


def attn_fwd_bwd_torch(q, k, v, do, cos, sin, has_cls: bool = True):
    """The "PyTorch SDPA + Python 2D RoPE" harness of README.md:123-136, restated.

    ``q, k, v, do`` are CPU torch tensors (any float dtype); the rotation uses
    the pair tables exactly as fa_rope_full .py:201-202. Returns
    ``(o, dq, dk, dv)``. This is also the timed CPU baseline.
    """
    import torch
    import torch.nn.functional as F

    N = q.shape[-2]
    off = 1 if has_cls else 0
    cos_t = torch.as_tensor(cos, dtype=q.dtype)
    sin_t = torch.as_tensor(sin, dtype=q.dtype)
    C = torch.ones(N, cos_t.shape[1], dtype=q.dtype)
    S = torch.zeros(N, cos_t.shape[1], dtype=q.dtype)
    C[off:] = cos_t[: N - off]
    S[off:] = sin_t[: N - off]

    def rot(x):
        e, o = x[..., 0::2], x[..., 1::2]
        return torch.stack((e * C - o * S, o * C + e * S), dim=-1).flatten(-2)

    q = q.detach().requires_grad_(True)
    k = k.detach().requires_grad_(True)
    v = v.detach().requires_grad_(True)
    o = F.scaled_dot_product_attention(rot(q), rot(k), v)
    o.backward(do)
    return o.detach(), q.grad, k.grad, v.grad


def flops_fwd_bwd(B: int, H: int, N: int, D: int) -> float:
    """Algorithmic FLOPs of one fwd+bwd: 4 (fwd) + 10 (bwd) N^2 D per head."""
    return 14.0 * B * H * N * N * D


def min_bytes_fwd_bwd(B: int, H: int, N: int, D: int, elt: int) -> float:
    """Minimum HBM bytes of one fwd+bwd: 12 [B,H,N,D] tensors plus LSE/Delta traffic."""
    return 12.0 * B * H * N * D * elt + 3.0 * B * H * N * 4
