"""The allocation-free backward (frsa_bwd_noalloc) against the regular one.

frsa_bwd_noalloc exists for callers that cannot allocate device memory (plugin
hosts that only pass in their input and output buffers, pre-carved memory
pools, loops that must not call cudaMalloc/cudaFree because those can
synchronise the device). It keeps its f32 dQ accumulator in a fixed array
inside the library instead of a caller-provided workspace. This file calls it
through the C ABI, twice in a row (the array keeps the previous call's
contents, so the second call checks that each call clears what it uses), and
compares dQ, dK, dV with frsa_bwd and with the float64 oracle under the parity
bar of the other GPU tests.

Named so pytest collects it last; it also passes when run alone.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import attn_bwd_np
from tests.helpers import MAX_ABS_TOL, MEAN_ABS_TOL, err_stats, seeded_inputs

pytestmark = pytest.mark.gpu


def _call_noalloc(q, k, v, o, lse, do, cosp, sinp, has_cls):
    from triton_fused_rope_flash_attn_b200 import _lib
    from triton_fused_rope_flash_attn_b200.attention import _make_args
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    a = _make_args(q, k, v, cosp, sinp, has_cls, q.dtype, o=o, lse=lse, d_o=do, dq=dq, dk=dk,
                   dv=dv)
    rc = _lib.load().frsa_bwd_noalloc(ctypes.byref(a),
                                     torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "frsa_bwd_noalloc")
    return dq, dk, dv


@pytest.mark.parametrize("B,H,side,has_cls,D,dtype", [
    (2, 4, 14, True, 64, torch.bfloat16),    # regular path: on-chip dQ
    (1, 3, 16, True, 64, torch.bfloat16),    # regular path: workspace
    (1, 2, 7, True, 80, torch.bfloat16),
    (1, 3, 16, True, 64, torch.float16)])
def test_noalloc_matches_regular_backward_twice(B, H, side, has_cls, D, dtype):
    from triton_fused_rope_flash_attn_b200 import (CosSinTable, _lib, fused_rope_attention_bwd,
                                                   fused_rope_attention_fwd)
    N = side * side + int(has_cls)
    cs = CosSinTable(100.0, side, D, device="cuda")
    for call in range(2):
        q, k, v, do = (t.cuda().to(dtype) for t in seeded_inputs(B, H, N, D, seed=11 + call))
        o, lse = fused_rope_attention_fwd(q, k, v, cs.COSP, cs.SINP, has_cls)
        ref = fused_rope_attention_bwd(q, k, v, o, lse, do, cs.COSP, cs.SINP, has_cls)
        got = _call_noalloc(q, k, v, o, lse, do, cs.COSP, cs.SINP, has_cls)
        torch.cuda.synchronize()
        assert _lib.load().frsa_query_status() == 0
        for name, g, r in zip(("dq", "dk", "dv"), got, ref):
            gn, rn = g.double().cpu().numpy(), r.double().cpu().numpy()
            assert np.isfinite(gn).all(), name
            mx, mean = err_stats(gn, rn)
            assert mx <= MAX_ABS_TOL and mean <= MEAN_ABS_TOL, (call, name, mx, mean)
        # and against the float64 oracle on the same quantised inputs
        cos, sin = cs.COSP.cpu().numpy(), cs.SINP.cpu().numpy()
        exact = attn_bwd_np(*(t.double().cpu().numpy() for t in (q, k, v, do)), cos, sin,
                            has_cls)
        for name, g, r in zip(("dq", "dk", "dv"), got, exact):
            mx, mean = err_stats(g.double().cpu().numpy(), r)
            assert mx <= MAX_ABS_TOL and mean <= MEAN_ABS_TOL, ("oracle", call, name, mx, mean)


def test_noalloc_rejects_float32():
    """Only 16-bit compute: float32 tensors are refused before anything launches."""
    from triton_fused_rope_flash_attn_b200 import CosSinTable, _lib
    from triton_fused_rope_flash_attn_b200.attention import _make_args
    cs = CosSinTable(100.0, 4, 64, device="cuda")
    q = torch.zeros(1, 1, 17, 64, device="cuda")
    lse = torch.zeros(1, 1, 17, device="cuda")
    a = _make_args(q, q, q, cs.COSP, cs.SINP, True, torch.float32, o=q, lse=lse, d_o=q, dq=q,
                   dk=q, dv=q)
    assert _lib.load().frsa_bwd_noalloc(ctypes.byref(a), None) == 4    # UNSUPPORTED_DTYPE


def test_noalloc_rejects_oversize():
    """A shape beyond the built-in scratch is refused before anything launches."""
    from triton_fused_rope_flash_attn_b200 import _lib
    lib = _lib.load()
    limit = lib.frsa_bwd_noalloc_max_elements()
    D, N = 64, 197
    H = limit // (N * D) + 1            # one head more than fits
    a = _lib.FrsaAttnArgs()
    dummy = torch.empty(16, device="cuda", dtype=torch.bfloat16)
    tab = torch.zeros(196, 32, device="cuda")
    for f in ("q", "k", "v", "o", "d_o", "dq", "dk", "dv"):
        setattr(a, f, dummy.data_ptr())
    a.lse = dummy.data_ptr()
    a.cosp, a.sinp = tab.data_ptr(), tab.data_ptr()
    a.B, a.H, a.N, a.D, a.n_pos, a.has_cls = 1, H, N, D, 196, 1
    a.io_dtype = a.compute_dtype = _lib.FRSA_DTYPE_BF16
    a.scale = 0.125
    rc = lib.frsa_bwd_noalloc(ctypes.byref(a), None)
    assert rc == 10, lib.frsa_strerror(rc)
    assert b"scratch" in lib.frsa_strerror(rc)
