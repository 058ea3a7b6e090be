"""Host-side contract tests that need no GPU: the reference's assertions and
error types, the compute-dtype rule, and the C-ABI library's exports and
argument validation (only calls that return before touching a device)."""
from __future__ import annotations

import ctypes
import os
import re

import pytest
import torch

import fa_rope_full
from triton_fused_rope_flash_attn_b200 import (CosSinTable, TritonAttention, _lib,
                                               _sdpa_comp_dtype, sdpa_triton_fa_rope)
from triton_fused_rope_flash_attn_b200.build import INCLUDE, build_library


@pytest.fixture(scope="module")
def lib():
    build_library()
    return _lib.load()


def test_dropin_module_exports():
    for name in ("build_axial_rope_pairs", "CosSinTable", "_sdpa_comp_dtype", "TritonAttention",
                 "sdpa_triton_fa_rope"):
        assert hasattr(fa_rope_full, name)


def test_comp_dtype_rule():
    x = torch.zeros(1, dtype=torch.float32)
    assert _sdpa_comp_dtype(x) == torch.float32
    assert _sdpa_comp_dtype(x.bfloat16()) == torch.bfloat16
    assert _sdpa_comp_dtype(x.half()) == torch.float16
    with pytest.raises(TypeError):
        _sdpa_comp_dtype(x.double())


@pytest.mark.parametrize("N,has_cls,msg", [
    (196, True, "SEQ_LEN must be 1 + H_img*W_img when has_cls=True (got 196 vs 197)."),
    (197, False, "SEQ_LEN must equal H_img*W_img when has_cls=False (got 197 vs 196)."),
])
def test_seq_len_assertions(N, has_cls, msg):
    q = torch.zeros(1, 1, N, 64)
    cs = CosSinTable(100.0, 14, 64, device="cpu")
    with pytest.raises(AssertionError, match=re.escape(msg)):
        TritonAttention.apply(q, q, q, cs, 14, has_cls)


def test_head_dim_assertion():
    q = torch.zeros(1, 1, 197, 62)
    cs = CosSinTable(100.0, 14, 64, device="cpu")
    with pytest.raises(AssertionError, match="HEAD_DIM must be divisible by 4"):
        sdpa_triton_fa_rope(q, q, q, cs)


def test_cpu_tensors_fail_loudly():
    """No CPU fallback: CPU inputs raise instead of computing."""
    q = torch.zeros(1, 1, 197, 64)
    cs = CosSinTable(100.0, 14, 64, device="cpu")
    with pytest.raises(RuntimeError, match="CUDA"):
        sdpa_triton_fa_rope(q, q, q, cs)


def test_header_symbols_exported(lib):
    with open(os.path.join(INCLUDE, "frsa.h")) as f:
        hdr = f.read()
    declared = set(re.findall(r"^\w[\w\s\*]*?\b(frsa_\w+)\(", hdr, flags=re.M))
    assert declared == set(_lib.EXPORTED_SYMBOLS)
    for name in declared:
        assert hasattr(lib, name), name
    assert lib.frsa_abi_version() == 2


def test_strerror_covers_codes(lib):
    for code in range(0, 11):
        msg = lib.frsa_strerror(code).decode()
        assert msg and "unknown" not in msg, code
    assert "unknown" in lib.frsa_strerror(99).decode()


def _args(**kw):
    a = _lib.FrsaAttnArgs()
    a.q = a.k = a.v = a.o = a.lse = 0x1000
    a.cosp = a.sinp = 0x2000
    a.B, a.H, a.N, a.D, a.n_pos, a.has_cls = 1, 1, 197, 64, 196, 1
    a.io_dtype = a.compute_dtype = _lib.FRSA_DTYPE_BF16
    a.scale = 0.125
    for k, v in kw.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize("kw,code", [
    (dict(q=None), 1),
    (dict(D=60), 3),
    (dict(D=136), 3),
    (dict(N=198), 2),               # table has 196 rows, N - has_cls = 197
    (dict(has_cls=2), 2),
    (dict(B=0), 2),
    (dict(io_dtype=_lib.FRSA_DTYPE_F32, compute_dtype=_lib.FRSA_DTYPE_BF16), 4),
    (dict(io_dtype=_lib.FRSA_DTYPE_F16, compute_dtype=_lib.FRSA_DTYPE_F32), 4),
    # float32 in and out (TF32 compute) is a valid forward: it gets as far as
    # the device check on a machine without an sm_100 GPU.
    (dict(io_dtype=_lib.FRSA_DTYPE_F32, compute_dtype=_lib.FRSA_DTYPE_F32), 8),
    (dict(k=0x1008), 5),
])
def test_fwd_validation_before_device(lib, kw, code):
    assert lib.frsa_fwd(ctypes.byref(_args(**kw)), None) == code


def test_bwd_float32_contract(lib):
    # float32 backward: D <= 64, a Delta workspace of B*H*N floats unless delta is given.
    a = _args(io_dtype=_lib.FRSA_DTYPE_F32, compute_dtype=_lib.FRSA_DTYPE_F32)
    a.d_o = a.dq = a.dk = a.dv = 0x3000
    assert lib.frsa_bwd_workspace_bytes(ctypes.byref(a)) == 197 * 4
    assert lib.frsa_bwd(ctypes.byref(a), None) == 9          # workspace missing
    a.workspace, a.workspace_bytes = 0x4000, 197 * 4
    assert lib.frsa_bwd(ctypes.byref(a), None) == 8          # no sm_100 device here
    a.delta = 0x5000
    assert lib.frsa_bwd_workspace_bytes(ctypes.byref(a)) == 0   # caller's delta: no scratch
    big = _args(io_dtype=_lib.FRSA_DTYPE_F32, compute_dtype=_lib.FRSA_DTYPE_F32, D=80, n_pos=196)
    big.d_o = big.dq = big.dk = big.dv = 0x3000
    assert lib.frsa_bwd(ctypes.byref(big), None) == 3        # D > 64: unsupported


def test_bwd_requires_gradients_and_workspace(lib):
    a = _args()
    assert lib.frsa_bwd(ctypes.byref(a), None) == 1              # no d_o / dq / dk / dv
    big = _args(N=257, n_pos=256, d_o=0x1000, dq=0x1000, dk=0x1000, dv=0x1000)
    # ABI 2: S = min(T, 8) partial slots of B*H*N*D floats (T = 3 key tiles here),
    # counters ((B*H*T*(1 + S) + 4) & ~3 int32), the rotated Q and K (16-bit) and
    # Delta rows (B*H*N floats, only without a caller `delta`).
    T = S = 3
    counters = ((1 * 1 * T * (1 + S) + 4) & ~3) * 4
    part = S * 257 * 64 * 4 + 2 * 257 * 64 * 2        # + rotated Q and K (bf16)
    assert lib.frsa_bwd_workspace_bytes(ctypes.byref(big)) == part + counters + 257 * 4
    big.delta = 0x2000
    assert lib.frsa_bwd_workspace_bytes(ctypes.byref(big)) == part + counters
    assert lib.frsa_bwd(ctypes.byref(big), None) == 9            # workspace missing
    big.workspace, big.workspace_bytes = 0x4000, part + counters
    assert lib.frsa_bwd(ctypes.byref(big), None) == 8            # enough: no sm_100 device here
    small = _args(d_o=0x1000, dq=0x1000, dk=0x1000, dv=0x1000)
    assert lib.frsa_bwd_workspace_bytes(ctypes.byref(small)) == 0


def test_table_shape_checked_by_wrapper():
    from triton_fused_rope_flash_attn_b200.attention import _check_tables
    c = torch.zeros(196, 32)
    _check_tables(c, c, 197, 64, True, c.device)
    with pytest.raises(ValueError):
        _check_tables(c, c, 198, 64, True, c.device)
    with pytest.raises(ValueError):
        _check_tables(c[:, :16], c[:, :16], 197, 64, True, c.device)
    with pytest.raises(TypeError):
        _check_tables(c.double(), c.double(), 197, 64, True, c.device)


def test_torch_extension_builds_binds_and_rejects_cpu_tensors():
    """The PyTorch C++ extension (the product path's host side) loads, binds the
    C ABI of libfrsa.so and refuses CPU tensors (there is no CPU path)."""
    from triton_fused_rope_flash_attn_b200.attention import _ext, fused_rope_attention_fwd
    ext = _ext()
    assert hasattr(ext, "fwd") and hasattr(ext, "bwd")
    q = torch.zeros(1, 1, 5, 64)
    tab = torch.zeros(4, 32)
    with pytest.raises(RuntimeError, match="CUDA"):
        fused_rope_attention_fwd(q, q, q, tab, tab, True)


def test_strides_and_flags_validated(lib):
    """q/k/v strides (b, h, n in elements) must be positive multiples of 16
    bytes; unknown flag bits are refused; FRSA_FLAG_NO_ROPE needs no tables."""
    def code(a):
        return lib.frsa_fwd(ctypes.byref(a), None)

    ok = _args(H=2)
    ok.q_strides[:] = [197 * 3 * 2 * 64, 64, 3 * 2 * 64]   # a [B, N, 3, H, D] view
    assert code(ok) == 8                                    # valid: no sm_100 device here
    bad = _args(H=2)
    bad.q_strides[:] = [197 * 3 * 2 * 64, 60, 3 * 2 * 64]  # 120-byte head stride
    assert code(bad) == 5
    neg = _args()
    neg.k_strides[:] = [0, 0, -64]
    assert code(neg) == 5
    flags = _args(flags=2)
    assert code(flags) == 2
    norope = _args(flags=_lib.FRSA_FLAG_NO_ROPE, n_pos=0)
    norope.cosp = norope.sinp = None
    assert code(norope) == 8                                # tables not needed
    rope = _args(n_pos=0)
    rope.cosp = rope.sinp = None
    assert code(rope) == 1                                  # tables needed


def test_convert_and_qkv_bwd_validation(lib):
    """frsa_convert_in/out and frsa_qkv_rope_bwd reject bad arguments before
    touching a device (codes from include/frsa.h)."""
    buf = (ctypes.c_uint8 * 4096)()
    p = ctypes.addressof(buf) + (-ctypes.addressof(buf)) % 256   # 256-byte aligned host stand-in

    def conv(**kw):
        a = _lib.FrsaConvertArgs()
        a.q = a.k = a.v = a.q_out = a.k_out = a.v_out = a.cosp = a.sinp = p
        a.B, a.H, a.N, a.D, a.n_pos, a.has_cls = 1, 2, 197, 64, 196, 1
        a.dtype = _lib.FRSA_DTYPE_BF16
        for k, v in kw.items():
            setattr(a, k, v)
        return a

    for fn in (lib.frsa_convert_in, lib.frsa_convert_out):
        assert fn(None, None) == 1                        # NULL_ARG
        assert fn(ctypes.byref(conv(q=None)), None) == 1
        assert fn(ctypes.byref(conv(N=0)), None) == 2     # BAD_SHAPE
        assert fn(ctypes.byref(conv(n_pos=100)), None) == 2   # table shorter than the tokens
        assert fn(ctypes.byref(conv(D=36)), None) == 3    # UNSUPPORTED_D
        assert fn(ctypes.byref(conv(dtype=_lib.FRSA_DTYPE_F32)), None) == 4
        assert fn(ctypes.byref(conv(q=p + 8)), None) == 5     # MISALIGNED

    def qb(**kw):
        a = _lib.FrsaQkvBwdArgs()
        a.dq = a.dk = a.dv = a.cosp = a.sinp = a.dqkv = p
        a.B, a.N, a.C, a.H, a.n_pos, a.has_cls = 1, 197, 768, 12, 196, 1
        a.dtype = _lib.FRSA_DTYPE_BF16
        for k, v in kw.items():
            setattr(a, k, v)
        return a

    assert lib.frsa_qkv_rope_bwd(None, None) == 1
    assert lib.frsa_qkv_rope_bwd(ctypes.byref(qb(dqkv=None)), None) == 1
    assert lib.frsa_qkv_rope_bwd(ctypes.byref(qb(C=770)), None) == 2     # C % H != 0
    assert lib.frsa_qkv_rope_bwd(ctypes.byref(qb(C=384, H=16)), None) == 3   # D = 24
    assert lib.frsa_qkv_rope_bwd(ctypes.byref(qb(dtype=_lib.FRSA_DTYPE_F32)), None) == 4
    assert lib.frsa_qkv_rope_bwd(ctypes.byref(qb(dq=p + 4)), None) == 5
