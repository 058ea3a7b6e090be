"""Autograd wrapper and public entry of the fused 2D-RoPE attention.

Mirrors ``TritonAttention`` / ``sdpa_triton_fa_rope`` of the reference
(fa_rope_full .py:1011-1170): the same assertions and messages, the same
output-dtype rule (outputs and gradients in the input dtype, compute in the
autocast dtype when CUDA autocast is on), ``scale = 1/sqrt(D)``, no mask. The
work is done by the C ABI (``include/frsa.h``) on torch's current stream.
"""
from __future__ import annotations

import math

import torch

from . import _lib

_DT_CODE = {torch.bfloat16: _lib.FRSA_DTYPE_BF16, torch.float16: _lib.FRSA_DTYPE_F16,
            torch.float32: _lib.FRSA_DTYPE_F32}


def _sdpa_comp_dtype(x: torch.Tensor) -> torch.dtype:
    """Compute dtype: the CUDA autocast dtype when autocast is on, else ``x.dtype``.

    fa_rope_full .py:65-73. The reference returns the matching Triton dtype and
    raises ``TypeError`` for anything but float16/bfloat16/float32; this returns
    the torch dtype and raises ``TypeError`` for the same cases.
    """
    dtype = torch.get_autocast_dtype("cuda") if torch.is_autocast_enabled() else x.dtype
    if dtype in (torch.float16, torch.bfloat16, torch.float32):
        return dtype
    raise TypeError(f"unsupported compute dtype {dtype}")


def _ptr(t):
    return None if t is None else t.data_ptr()


def _make_args(q, k, v, cosp, sinp, has_cls, comp, o=None, lse=None, d_o=None, dq=None, dk=None,
               dv=None, delta=None, workspace=None, scale=None):
    B, H, N, D = q.shape
    a = _lib.FrsaAttnArgs()
    a.q, a.k, a.v = _ptr(q), _ptr(k), _ptr(v)
    a.o, a.lse = _ptr(o), _ptr(lse)
    a.d_o, a.dq, a.dk, a.dv, a.delta = _ptr(d_o), _ptr(dq), _ptr(dk), _ptr(dv), _ptr(delta)
    a.workspace = _ptr(workspace)
    a.workspace_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    a.cosp, a.sinp = _ptr(cosp), _ptr(sinp)
    a.B, a.H, a.N, a.D = B, H, N, D
    a.n_pos = cosp.shape[0]
    a.has_cls = int(bool(has_cls))
    a.io_dtype = _DT_CODE[comp]
    a.compute_dtype = _DT_CODE[comp]
    a.scale = 1.0 / math.sqrt(D) if scale is None else float(scale)
    return a


def _check_tables(cosp, sinp, N, D, has_cls, device):
    if cosp.dtype != torch.float32 or sinp.dtype != torch.float32:
        raise TypeError("COSP/SINP must be float32")
    if cosp.dim() != 2 or cosp.shape[1] != D // 2 or sinp.shape != cosp.shape:
        raise ValueError(f"COSP/SINP must be [N_pos, {D // 2}], got {tuple(cosp.shape)} / "
                         f"{tuple(sinp.shape)}")
    if cosp.shape[0] < N - int(bool(has_cls)):
        raise ValueError(f"RoPE table has {cosp.shape[0]} positions, sequence needs "
                         f"{N - int(bool(has_cls))}")
    if cosp.device != device or sinp.device != device:
        raise ValueError("RoPE tables must be on the same device as Q")


_EXT = None


def _ext():
    """The PyTorch C++ extension (``csrc/frsa_torch.cpp``), bound to the loaded C ABI.

    Built in-tree on first use if missing; there is no fallback path.
    """
    global _EXT
    if _EXT is None:
        import ctypes
        from .build import build_torch_ext
        lib = _lib.load()
        if lib.frsa_abi_version() != 2:
            raise RuntimeError(f"libfrsa.so ABI version {lib.frsa_abi_version()}, expected 2")
        ext = build_torch_ext()
        addr = lambda f: ctypes.cast(f, ctypes.c_void_p).value  # noqa: E731
        ext.bind(addr(lib.frsa_fwd), addr(lib.frsa_bwd), addr(lib.frsa_bwd_workspace_bytes))
        _EXT = ext
    return _EXT


_NO_TABLE = {}


def _tables_or_placeholder(cosp, sinp, rope, device):
    if rope:
        return cosp, sinp
    if device not in _NO_TABLE:
        _NO_TABLE[device] = torch.empty(0, device=device, dtype=torch.float32)
    return _NO_TABLE[device], _NO_TABLE[device]


def fused_rope_attention_fwd(q, k, v, cosp, sinp, has_cls: bool = True, scale=None,
                             rope: bool = True):
    """Forward through the C ABI. ``q, k, v``: CUDA ``[B, H, N, D]``, all bf16, f16 or f32
    (any b/h/n strides that are multiples of 16 bytes are read in place).

    Returns ``(o, lse)`` with ``lse`` float32 ``[B, H, N]`` (natural log).
    ``scale`` multiplies the logits (default ``1/sqrt(D)``). ``rope=False``:
    q and k are already rotated (the tables are not used and may be None).
    """
    cosp, sinp = _tables_or_placeholder(cosp, sinp, rope, q.device)
    o, lse, rc = _ext().fwd(q, k, v, cosp, sinp, bool(has_cls), -1.0 if scale is None else scale,
                            0 if rope else _lib.FRSA_FLAG_NO_ROPE)
    _lib.check(rc, "frsa_fwd")
    return o, lse


def fused_rope_attention_bwd(q, k, v, o, lse, d_o, cosp, sinp, has_cls: bool = True,
                             delta_out=None, scale=None, rope: bool = True):
    """Backward through the C ABI. Returns ``(dq, dk, dv)`` in ``q.dtype``.

    ``delta_out`` (optional float32 ``[B, H, N]``) receives ``rowsum(dO * O)``.
    ``rope=False``: q and k are already rotated and dq, dk are the gradients
    with respect to them.
    """
    cosp, sinp = _tables_or_placeholder(cosp, sinp, rope, q.device)
    dq, dk, dv, rc = _ext().bwd(q, k, v, o, lse, d_o, cosp, sinp, bool(has_cls), delta_out,
                                -1.0 if scale is None else scale,
                                0 if rope else _lib.FRSA_FLAG_NO_ROPE)
    _lib.check(rc, "frsa_bwd")
    return dq, dk, dv


def _pow2_normaliser(x: torch.Tensor, target: float = 1.0) -> float:
    """Power of two s with max|x * s| <= target (1 for an all-zero tensor)."""
    m = float(x.detach().abs().max()) if x.numel() else 0.0
    if not math.isfinite(m):
        raise FloatingPointError("non-finite input to the fused attention")
    if m == 0.0:
        return 1.0
    return 2.0 ** math.floor(math.log2(target / m))


# float32 compute. The reference computes fp32 inputs with Triton's TF32 dot
# products (10-bit mantissa operands, fp32 accumulation; fa_rope_full .py:65-73
# selects float32 as the kernel dtype). Here the forward, and the backward for
# D <= 64, are native kind::tf32 kernels (fp32 in and out). For D > 64 the
# backward runs on the f16 kernels, whose operands have the same 10-bit
# mantissa as TF32, with accumulation in fp32; f16's narrower exponent range is
# handled exactly: each operand is multiplied by a power of two that brings its
# largest magnitude to 1 (dO to 1/8, leaving headroom for dV = P^T dO and
# dQ = dS K), the logit scale absorbs the Q and K factors, and the gradients
# are divided back and returned in fp32.
def _fp32_forward(Q, K, V, COSP, SINP, has_cls, rope=True):
    return fused_rope_attention_fwd(Q.contiguous(), K.contiguous(), V.contiguous(), COSP, SINP,
                                    has_cls, rope=rope)


def _fp32_backward(Q, K, V, O, lse, dO, COSP, SINP, has_cls, rope=True):
    D = Q.shape[-1]
    if D <= 64:
        return fused_rope_attention_bwd(Q, K, V, O, lse, dO.contiguous(), COSP, SINP, has_cls,
                                        rope=rope)
    sq, sk, sv = _pow2_normaliser(Q), _pow2_normaliser(K), _pow2_normaliser(V)
    sd = _pow2_normaliser(dO, 0.125)
    qh, kh, vh = (Q * sq).half(), (K * sk).half(), (V * sv).half()
    oh, doh = (O * sv).half(), (dO * sd).half()
    scale = 1.0 / math.sqrt(D) / (sq * sk)
    dq, dk, dv = fused_rope_attention_bwd(qh, kh, vh, oh, lse, doh, COSP, SINP, has_cls,
                                          scale=scale, rope=rope)
    dq = dq.float() * (sq / (sd * sv))
    dk = dk.float() * (sk / (sd * sv))
    dv = dv.float() / sd
    for g in (dq, dk, dv):
        if not torch.isfinite(g).all():
            raise FloatingPointError("float32 attention gradient left the f16 operand range")
    return dq, dk, dv


def _convert(to_16bit, srcs, dsts, COSP, SINP, has_cls, comp):
    """frsa_convert_in (f32 q, k, v -> rotated 16-bit) or frsa_convert_out
    (16-bit dq^, dk^, dv -> f32 with R^T) on torch's current stream."""
    B, H, N, D = srcs[0].shape
    a = _lib.FrsaConvertArgs()
    a.q, a.k, a.v = (t.data_ptr() for t in srcs)
    a.q_out, a.k_out, a.v_out = (t.data_ptr() for t in dsts)
    a.cosp, a.sinp = COSP.data_ptr(), SINP.data_ptr()
    a.B, a.H, a.N, a.D, a.n_pos = B, H, N, D, COSP.shape[0]
    a.has_cls = int(bool(has_cls))
    a.dtype = _DT_CODE[comp]
    lib = _lib.load()
    fn = lib.frsa_convert_in if to_16bit else lib.frsa_convert_out
    _lib.check(fn(a, torch.cuda.current_stream(srcs[0].device).cuda_stream),
               "frsa_convert_in" if to_16bit else "frsa_convert_out")


class TritonAttention(torch.autograd.Function):
    """Fused 2D-RoPE SDPA with the reference's autograd contract (fa_rope_full .py:1011-1138)."""

    @staticmethod
    def forward(ctx, Q, K, V, cos_sin, H_img=14, has_cls=True, rope=True):
        BATCH_SIZE, NUM_HEADS, SEQ_LEN, HEAD_DIM = Q.size()
        assert (HEAD_DIM % 4) == 0, "HEAD_DIM must be divisible by 4 (2D RoPE requires pairs)."
        N_img = H_img ** 2
        if has_cls:
            assert SEQ_LEN == 1 + N_img, (
                f"SEQ_LEN must be 1 + H_img*W_img when has_cls=True (got {SEQ_LEN} vs {1+N_img}).")
        else:
            assert SEQ_LEN == N_img, (
                f"SEQ_LEN must equal H_img*W_img when has_cls=False (got {SEQ_LEN} vs {N_img}).")
        comp = _sdpa_comp_dtype(Q)
        if not Q.is_cuda:
            raise RuntimeError("sdpa_triton_fa_rope needs CUDA tensors (there is no CPU path)")
        if rope:
            COSP, SINP = cos_sin.tables()
            _check_tables(COSP, SINP, SEQ_LEN, HEAD_DIM, has_cls, Q.device)
        else:   # q and k arrive rotated: no tables
            COSP, SINP = _tables_or_placeholder(None, None, False, Q.device)
        ctx.comp = comp
        ctx.has_cls = has_cls
        ctx.rope = rope
        ctx.io_dtypes = (Q.dtype, K.dtype, V.dtype)
        ctx.convert = False
        if comp == torch.float32:
            Qf, Kf, Vf = (t.float().contiguous() for t in (Q, K, V))
            o, lse = _fp32_forward(Qf, Kf, Vf, COSP, SINP, has_cls, rope)
            ctx.save_for_backward(Qf, Kf, Vf, o, lse, COSP, SINP)
            return o.to(Q.dtype)
        ctx.convert = (rope and Q.dtype == K.dtype == V.dtype == torch.float32
                       and HEAD_DIM % 8 == 0)
        if ctx.convert:
            # f32 inputs, 16-bit compute: one kernel converts q, k, v and
            # applies the rotation (in f32, one rounding); the attention then
            # rotates nothing, and the backward converts the gradients back.
            Qf, Kf, Vf = (t.contiguous() for t in (Q, K, V))
            qc, kc, vc = (torch.empty(Q.shape, device=Q.device, dtype=comp) for _ in range(3))
            _convert(True, (Qf, Kf, Vf), (qc, kc, vc), COSP, SINP, has_cls, comp)
            o, lse = fused_rope_attention_fwd(qc, kc, vc, None, None, has_cls, rope=False)
            ctx.save_for_backward(qc, kc, vc, o, lse, COSP, SINP)
            return o.to(Q.dtype)
        qc, kc, vc = (t.to(comp) for t in (Q, K, V))
        o, lse = fused_rope_attention_fwd(qc, kc, vc, COSP, SINP, has_cls, rope=rope)
        ctx.save_for_backward(qc, kc, vc, o, lse, COSP, SINP)
        return o.to(Q.dtype)

    @staticmethod
    def backward(ctx, dO):
        qc, kc, vc, o, lse, COSP, SINP = ctx.saved_tensors
        if ctx.comp == torch.float32:
            dq, dk, dv = _fp32_backward(qc, kc, vc, o, lse, dO.float(), COSP, SINP, ctx.has_cls,
                                        ctx.rope)
        elif ctx.convert:
            gq, gk, gv = fused_rope_attention_bwd(qc, kc, vc, o, lse, dO.to(ctx.comp), None, None,
                                                  ctx.has_cls, rope=False)
            dq, dk, dv = (torch.empty(qc.shape, device=qc.device, dtype=torch.float32)
                          for _ in range(3))
            _convert(False, (gq, gk, gv), (dq, dk, dv), COSP, SINP, ctx.has_cls, ctx.comp)
        else:
            dq, dk, dv = fused_rope_attention_bwd(qc, kc, vc, o, lse, dO.to(ctx.comp), COSP, SINP,
                                                  ctx.has_cls, rope=ctx.rope)
        qd, kd, vd = ctx.io_dtypes
        return dq.to(qd), dk.to(kd), dv.to(vd), None, None, None, None


def sdpa_triton_fa_rope(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, cos_sin, *,
                        has_cls: bool = True, H_img: int | None = None, rope: bool = True):
    """Fused 2D-RoPE SDPA forward; differentiable (fa_rope_full .py:1169-1170).

    With the reference's four positional arguments this behaves like the
    reference. ``has_cls``, ``H_img`` and ``rope`` are keyword extensions;
    ``H_img`` defaults to the side of ``cos_sin``'s table (14 for the
    reference's 14x14 grid). ``rope=False``: Q and K are already rotated (for
    example by the fused QKV projection), nothing is rotated and the Q/K
    gradients are with respect to the given tensors; ``cos_sin`` may be None
    (then ``H_img`` must be given).
    """
    if H_img is None:
        n_pos = cos_sin.tables()[0].shape[0]
        H_img = math.isqrt(n_pos)
    return TritonAttention.apply(Q, K, V, cos_sin, H_img, has_cls, rope)
