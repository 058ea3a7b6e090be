"""GPU parity: the sm_100a kernels (through the C ABI) against the float64 oracle.

Inputs are seeded, quantised to the compute dtype, and the oracle is evaluated
in float64 on exactly those quantised values with the same float32 tables.
Bar: max abs error <= 3e-2 and mean abs error <= 1e-3 on O, dQ, dK, dV (bf16;
for N < 16 the mean bound is max(1e-3, 2e-2 * mean|exact|): P and dS are O(1)
there and their bf16 rounding dominates);
LSE within 1e-2 abs. The ViT-H-like case (inputs x2.0, D=80) is checked by
relative error instead, because rounding the exact outputs to bf16 alone
exceeds the absolute mean bound there.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attn_bwd_np, attn_fwd_np
from tests.helpers import MAX_ABS_TOL, MEAN_ABS_TOL, err_stats, mean_tol, rel_err, seeded_inputs

pytestmark = pytest.mark.gpu

# (B, H, H_img, has_cls, D, amp, dtype)
CASES = [
    (1, 2, 1, True, 64, 1.0, torch.bfloat16),     # N=2
    (1, 2, 1, False, 64, 1.0, torch.bfloat16),    # N=1
    (1, 2, 2, True, 64, 1.0, torch.bfloat16),     # N=5
    (2, 1, 3, False, 64, 1.0, torch.bfloat16),    # N=9
    (1, 2, 5, True, 64, 1.0, torch.bfloat16),     # N=26
    (1, 2, 7, False, 64, 1.0, torch.bfloat16),    # N=49
    (1, 2, 7, True, 64, 1.0, torch.bfloat16),     # N=50
    (2, 3, 11, False, 64, 1.0, torch.bfloat16),   # N=121
    (2, 4, 14, True, 64, 1.0, torch.bfloat16),    # N=197 (ViT-S/B)
    (2, 4, 14, True, 64, 1.0, torch.float16),     # N=197 fp16
    (1, 3, 16, False, 64, 1.0, torch.bfloat16),   # N=256
    (1, 3, 16, True, 64, 1.0, torch.bfloat16),    # N=257 (general path: ordered dQ)
    (1, 3, 16, True, 64, 1.0, torch.float16),     # N=257 fp16 (Delta pre-pass for __half)
    (1, 2, 24, False, 64, 1.0, torch.bfloat16),   # N=576 (ViT-L)
    (1, 2, 14, True, 32, 1.0, torch.bfloat16),    # D=32
    (1, 2, 15, True, 48, 1.0, torch.bfloat16),    # D=48, N=226 (240 computed keys)
    (1, 2, 7, True, 80, 1.0, torch.bfloat16),     # D=80, N=50
    (1, 2, 7, True, 80, 1.0, torch.float16),      # D=80 fp16 (general path)
    (1, 2, 14, True, 128, 1.0, torch.bfloat16),   # D=128
]


def _run(B, H, side, has_cls, D, amp, dtype, seed=0):
    from triton_fused_rope_flash_attn_b200 import CosSinTable, fused_rope_attention_bwd, \
        fused_rope_attention_fwd
    N = side * side + (1 if has_cls else 0)
    q, k, v, do = seeded_inputs(B, H, N, D, amp, seed)
    dev = torch.device("cuda")
    cs = CosSinTable(100.0, side, D, device="cuda")
    qd, kd, vd, dod = (t.to(dev, dtype) for t in (q, k, v, do))
    o, lse = fused_rope_attention_fwd(qd, kd, vd, cs.COSP, cs.SINP, has_cls)
    dq, dk, dv = fused_rope_attention_bwd(qd, kd, vd, o, lse, dod, cs.COSP, cs.SINP, has_cls)
    torch.cuda.synchronize()
    from triton_fused_rope_flash_attn_b200 import _lib
    assert _lib.load().frsa_query_status() == 0
    cos, sin = cs.COSP.cpu().numpy(), cs.SINP.cpu().numpy()
    qn, kn, vn, don = (t.to(dtype).double().numpy() for t in (q, k, v, do))
    o_ref, lse_ref = attn_fwd_np(qn, kn, vn, cos, sin, has_cls)
    dq_ref, dk_ref, dv_ref = attn_bwd_np(qn, kn, vn, don, cos, sin, has_cls)
    got = {n: t.double().cpu().numpy() for n, t in (("o", o), ("lse", lse), ("dq", dq),
                                                     ("dk", dk), ("dv", dv))}
    ref = {"o": o_ref, "lse": lse_ref, "dq": dq_ref, "dk": dk_ref, "dv": dv_ref}
    return got, ref


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"B{c[0]}H{c[1]}s{c[2]}c{int(c[3])}D{c[4]}"
                         f"{'bf16' if c[6] == torch.bfloat16 else 'f16'}")
def test_fwd_bwd_parity(case):
    got, ref = _run(*case)
    N = case[2] ** 2 + int(case[3])
    for name in ("o", "dq", "dk", "dv"):
        assert np.isfinite(got[name]).all(), name
        mx, mean = err_stats(got[name], ref[name])
        assert mx <= MAX_ABS_TOL, f"{name}: max abs err {mx:.3e}"
        if N < 16:
            # Few keys: P and dS are O(1) and their bf16 rounding (which the
            # reference applies too, fa_rope_full .py:965) dominates the mean.
            bound = max(MEAN_ABS_TOL, 2e-2 * float(np.abs(ref[name]).mean()))
            assert mean <= bound, f"{name}: mean abs err {mean:.3e} > {bound:.3e}"
        else:
            assert mean <= mean_tol(ref[name], case[6]), f"{name}: mean abs err {mean:.3e}"
    mx, _ = err_stats(got["lse"], ref["lse"])
    assert mx <= 1e-2, f"lse max abs err {mx:.3e}"


@pytest.mark.parametrize("side,D", [(37, 80), (14, 64)])
def test_amplified_inputs_relative(side, D):
    """Inputs x2.0 (logits 4x wider, a peaked softmax): N=1370, D=80 (ViT-H
    like, general kernels) and N=197, D=64 (persistent kernels). The bf16
    rounding of the wider logits and outputs exceeds the absolute bar, so the
    bar is a relative mean error <= 1e-2 on every tensor."""
    got, ref = _run(1, 2, side, True, D, 2.0, torch.bfloat16)
    for name in ("o", "dq", "dk", "dv"):
        assert np.isfinite(got[name]).all(), name
        assert rel_err(got[name], ref[name]) <= 1e-2, name


def test_autograd_wrapper_matches_direct_calls():
    """TritonAttention.apply under bf16 autocast with fp32 leaves (README usage)."""
    from triton_fused_rope_flash_attn_b200 import CosSinTable, sdpa_triton_fa_rope
    B, H, side, D = 2, 2, 14, 64
    N = side * side + 1
    q, k, v, do = seeded_inputs(B, H, N, D)
    cs = CosSinTable(100.0, side, D, device="cuda")
    qd, kd, vd = (t.cuda().requires_grad_(True) for t in (q, k, v))
    with torch.autocast("cuda", dtype=torch.bfloat16):
        o = sdpa_triton_fa_rope(qd, kd, vd, cs)
    assert o.dtype == torch.float32
    o.backward(do.cuda())
    cos, sin = cs.COSP.cpu().numpy(), cs.SINP.cpu().numpy()
    qn, kn, vn = (t.bfloat16().double().numpy() for t in (q, k, v))
    o_ref, _ = attn_fwd_np(qn, kn, vn, cos, sin, True)
    dq_ref, dk_ref, dv_ref = attn_bwd_np(qn, kn, vn, do.bfloat16().double().numpy(), cos, sin,
                                         True)
    for got, r in ((o, o_ref), (qd.grad, dq_ref), (kd.grad, dk_ref), (vd.grad, dv_ref)):
        assert got.dtype == torch.float32
        mx, mean = err_stats(got.detach().double().cpu().numpy(), r)
        assert mx <= MAX_ABS_TOL and mean <= MEAN_ABS_TOL, (mx, mean)


def test_deterministic_resident_path():
    """N <= 256 reduces dQ on chip: two runs are bitwise identical."""
    from triton_fused_rope_flash_attn_b200 import CosSinTable, fused_rope_attention_bwd, \
        fused_rope_attention_fwd
    B, H, side, D = 2, 3, 14, 64
    N = side * side + 1
    q, k, v, do = (t.cuda().bfloat16() for t in seeded_inputs(B, H, N, D, seed=7))
    cs = CosSinTable(100.0, side, D, device="cuda")
    outs = []
    for _ in range(2):
        o, lse = fused_rope_attention_fwd(q, k, v, cs.COSP, cs.SINP, True)
        outs.append((o, lse) + fused_rope_attention_bwd(q, k, v, o, lse, do, cs.COSP, cs.SINP,
                                                        True))
    for a, b in zip(*outs):
        assert torch.equal(a, b)


@pytest.mark.parametrize("B,H,side,has_cls,D", [(4, 8, 24, False, 64),    # N=576: 5 key tiles
                                                (1, 4, 37, True, 80),     # N=1370, D=80: 11
                                                (2, 3, 16, True, 64)])    # N=257: 3 key tiles
def test_deterministic_general_path(B, H, side, has_cls, D):
    """N > 256 or D > 64: dQ is summed over key tiles in a fixed order, so
    repeated runs are bitwise identical even though CTAs claim work in
    whatever order they reach the ticket counter. A differently shaped call in
    between changes the timing of the next run."""
    from triton_fused_rope_flash_attn_b200 import CosSinTable, fused_rope_attention_bwd, \
        fused_rope_attention_fwd
    N = side * side + int(has_cls)
    q, k, v, do = (t.cuda().bfloat16() for t in seeded_inputs(B, H, N, D, seed=5))
    cs = CosSinTable(100.0, side, D, device="cuda")
    o, lse = fused_rope_attention_fwd(q, k, v, cs.COSP, cs.SINP, has_cls)
    first = fused_rope_attention_bwd(q, k, v, o, lse, do, cs.COSP, cs.SINP, has_cls)
    for rep in range(3):
        xs = torch.randn(3 + rep, 2, N, D, device="cuda").bfloat16()
        fused_rope_attention_bwd(xs, xs, xs, *fused_rope_attention_fwd(xs, xs, xs, cs.COSP,
                                                                       cs.SINP, has_cls),
                                 xs, cs.COSP, cs.SINP, has_cls)
        again = fused_rope_attention_bwd(q, k, v, o, lse, do, cs.COSP, cs.SINP, has_cls)
        for name, a, b in zip(("dq", "dk", "dv"), first, again):
            assert torch.equal(a, b), (rep, name)
    from triton_fused_rope_flash_attn_b200 import _lib
    torch.cuda.synchronize()
    assert _lib.load().frsa_query_status() == 0


@pytest.mark.parametrize("side,has_cls", [(14, True), (24, False)])
def test_delta_rowsum(side, has_cls):
    """The fused Delta = rowsum(dO * O) (fa_rope_full .py:352-357) in both backward modes."""
    from triton_fused_rope_flash_attn_b200 import CosSinTable, fused_rope_attention_bwd, \
        fused_rope_attention_fwd
    B, H, D = 1, 3, 64
    N = side * side + int(has_cls)
    q, k, v, do = (t.cuda().bfloat16() for t in seeded_inputs(B, H, N, D, seed=3))
    cs = CosSinTable(100.0, side, D, device="cuda")
    o, lse = fused_rope_attention_fwd(q, k, v, cs.COSP, cs.SINP, has_cls)
    delta = torch.full((B, H, N), float("nan"), device="cuda")
    fused_rope_attention_bwd(q, k, v, o, lse, do, cs.COSP, cs.SINP, has_cls, delta_out=delta)
    ref = (o.double() * do.double()).sum(-1)
    assert torch.allclose(delta.double(), ref, atol=1e-4, rtol=1e-4)


@pytest.mark.parametrize("side,has_cls,D,qamp,vamp", [(14, True, 64, 1.0, 1.0),
                                                      (5, False, 64, 1.0, 1000.0),
                                                      (7, True, 80, 2.0, 1e-3),
                                                      (17, True, 64, 1.0, 1.0)])
def test_fp32_compute_against_oracle(side, has_cls, D, qamp, vamp):
    """float32 inputs without autocast (the reference's TF32 mode): native TF32
    forward; backward on f16 operands (TF32's 10-bit mantissa) with power-of-two
    range scaling; fp32 outputs. Checked against the float64 oracle on the same
    fp32 inputs, relative to each output's scale, at 1e-2: both halves round
    every product operand to 10 mantissa bits (TF32 itself does), and the
    backward recomputes the logits from differently rounded operands than the
    forward's LSE. V and dO are scaled by `vamp` (1000x and 1e-3x: outside or at
    the edge of f16's range without the scaling); q by `qamp` (sharper softmax)."""
    from triton_fused_rope_flash_attn_b200 import CosSinTable, sdpa_triton_fa_rope
    B, H = 2, 2
    N = side * side + (1 if has_cls else 0)
    q, k, v, do = seeded_inputs(B, H, N, D, 1.0, 11)
    q, v, do = q * qamp, v * vamp, do * vamp
    cs = CosSinTable(100.0, side, D, device="cuda")
    qd, kd, vd = (t.cuda().float().requires_grad_(True) for t in (q, k, v))
    o = sdpa_triton_fa_rope(qd, kd, vd, cs, has_cls=has_cls, H_img=side)
    o.backward(do.cuda().float())
    assert o.dtype == torch.float32 and qd.grad.dtype == torch.float32
    cos, sin = cs.COSP.cpu().numpy(), cs.SINP.cpu().numpy()
    qn, kn, vn, don = (t.double().numpy() for t in (q, k, v, do))
    o_ref, _ = attn_fwd_np(qn, kn, vn, cos, sin, has_cls)
    dq_ref, dk_ref, dv_ref = attn_bwd_np(qn, kn, vn, don, cos, sin, has_cls)
    for name, got, ref in (("o", o, o_ref), ("dq", qd.grad, dq_ref), ("dk", kd.grad, dk_ref),
                           ("dv", vd.grad, dv_ref)):
        g = got.detach().double().cpu().numpy()
        err = np.abs(g - ref).max() / max(np.abs(ref).max(), 1e-30)
        assert err < 1e-2, (name, err)


@pytest.mark.parametrize("side,has_cls,D", [(14, True, 64), (3, False, 64), (16, True, 64),
                                            (7, True, 80), (5, False, 128), (6, True, 32)])
def test_tf32_forward_against_oracle(side, has_cls, D):
    """Native float32 forward (tcgen05 kind::tf32) through the C ABI. TF32 keeps
    10 mantissa bits of each operand, so the bar is relative: 5e-3 of the
    output scale (O); LSE within 1e-2 absolute."""
    from triton_fused_rope_flash_attn_b200 import CosSinTable, fused_rope_attention_fwd
    B, H = 2, 3
    N = side * side + (1 if has_cls else 0)
    q, k, v, _ = seeded_inputs(B, H, N, D, 1.0, 21)
    cs = CosSinTable(100.0, side, D, device="cuda")
    o, lse = fused_rope_attention_fwd(q.cuda().float(), k.cuda().float(), v.cuda().float(),
                                      cs.COSP, cs.SINP, has_cls)
    torch.cuda.synchronize()
    from triton_fused_rope_flash_attn_b200 import _lib
    assert _lib.load().frsa_query_status() == 0
    assert o.dtype == torch.float32
    cos, sin = cs.COSP.cpu().numpy(), cs.SINP.cpu().numpy()
    o_ref, lse_ref = attn_fwd_np(q.double().numpy(), k.double().numpy(), v.double().numpy(),
                                 cos, sin, has_cls)
    err = np.abs(o.double().cpu().numpy() - o_ref).max() / np.abs(o_ref).max()
    assert err < 5e-3, err
    assert np.abs(lse.double().cpu().numpy() - lse_ref).max() < 1e-2



@pytest.mark.parametrize("side,has_cls,D", [(14, True, 64), (3, False, 64), (16, True, 64),
                                            (6, True, 32), (24, False, 64)])
def test_tf32_backward_against_oracle(side, has_cls, D):
    """Native float32 backward (kind::tf32: Delta pass, dK/dV kernel, dQ kernel)
    through the C ABI, against the float64 oracle; bar 5e-3 of each output's scale."""
    from triton_fused_rope_flash_attn_b200 import (CosSinTable, fused_rope_attention_bwd,
                                                   fused_rope_attention_fwd)
    B, H = 2, 2
    N = side * side + (1 if has_cls else 0)
    q, k, v, do = seeded_inputs(B, H, N, D, 1.0, 23)
    cs = CosSinTable(100.0, side, D, device="cuda")
    qd, kd, vd, dod = (t.cuda().float() for t in (q, k, v, do))
    o, lse = fused_rope_attention_fwd(qd, kd, vd, cs.COSP, cs.SINP, has_cls)
    dq, dk, dv = fused_rope_attention_bwd(qd, kd, vd, o, lse, dod, cs.COSP, cs.SINP, has_cls)
    torch.cuda.synchronize()
    from triton_fused_rope_flash_attn_b200 import _lib
    assert _lib.load().frsa_query_status() == 0
    cos, sin = cs.COSP.cpu().numpy(), cs.SINP.cpu().numpy()
    refs = attn_bwd_np(q.double().numpy(), k.double().numpy(), v.double().numpy(),
                       do.double().numpy(), cos, sin, has_cls)
    for name, got, ref in zip(("dq", "dk", "dv"), (dq, dk, dv), refs):
        assert got.dtype == torch.float32
        err = np.abs(got.double().cpu().numpy() - ref).max() / np.abs(ref).max()
        assert err < 5e-3, (name, err)


@pytest.mark.parametrize("B,H,side,has_cls,D,dtype", [(2, 4, 14, True, 64, torch.bfloat16),
                                                      (1, 3, 24, False, 64, torch.bfloat16),
                                                      (1, 2, 7, True, 80, torch.float16)])
def test_strided_qkv_views_read_in_place(B, H, side, has_cls, D, dtype):
    """q, k, v as the [B, H, N, D] views of a [B, N, 3, H, D] projection output
    (the ViT block's layout; the reference accepts any strides, fa_rope_full
    .py:1043) are read through strided tensor maps: outputs and gradients are
    bitwise equal to those of contiguous copies."""
    from triton_fused_rope_flash_attn_b200 import CosSinTable, sdpa_triton_fa_rope
    N = side * side + int(has_cls)
    g = torch.Generator(device="cuda").manual_seed(3)
    qkv = torch.randn(B, N, 3, H, D, device="cuda", generator=g).to(dtype)
    do = torch.randn(B, H, N, D, device="cuda", generator=g).to(dtype)
    cs = CosSinTable(100.0, side, D, device="cuda")
    views = [x.detach().requires_grad_(True) for x in qkv.permute(2, 0, 3, 1, 4).unbind(0)]
    assert not views[0].is_contiguous()
    conts = [t.detach().contiguous().requires_grad_(True) for t in views]
    outs = []
    for q, k, v in (views, conts):
        o = sdpa_triton_fa_rope(q, k, v, cs, has_cls=has_cls, H_img=side)
        o.backward(do)
        outs.append((o.detach(), q.grad, k.grad, v.grad))
    for name, a, b in zip(("o", "dq", "dk", "dv"), *outs):
        assert torch.equal(a, b), name


@pytest.mark.parametrize("B,H,side,has_cls,D", [(2, 3, 14, True, 64), (1, 2, 24, False, 64),
                                                (1, 2, 7, True, 80)])
def test_no_rope_flag_equals_identity_tables(B, H, side, has_cls, D):
    """rope=False (FRSA_FLAG_NO_ROPE: q, k arrive rotated, nothing is rotated,
    gradients w.r.t. the given q, k) is bitwise the attention with identity
    tables, and matches the float64 oracle with identity tables."""
    from triton_fused_rope_flash_attn_b200 import sdpa_triton_fa_rope

    class Identity:
        def __init__(self, n_pos):
            self.c = torch.ones(n_pos, D // 2, device="cuda")
            self.s = torch.zeros(n_pos, D // 2, device="cuda")

        def tables(self):
            return self.c, self.s

    N = side * side + int(has_cls)
    q, k, v, do = (t.cuda().bfloat16() for t in seeded_inputs(B, H, N, D, seed=9))
    outs = []
    for rope, cs in ((True, Identity(side * side)), (False, None)):
        qd, kd, vd = (t.clone().requires_grad_(True) for t in (q, k, v))
        o = sdpa_triton_fa_rope(qd, kd, vd, cs, has_cls=has_cls, H_img=side, rope=rope)
        o.backward(do)
        outs.append((o.detach(), qd.grad, kd.grad, vd.grad))
    for name, a, b in zip(("o", "dq", "dk", "dv"), *outs):
        assert torch.equal(a, b), name
    ident = np.ones((side * side, D // 2), np.float32), np.zeros((side * side, D // 2), np.float32)
    qn, kn, vn, don = (t.double().cpu().numpy() for t in (q, k, v, do))
    refs = (attn_fwd_np(qn, kn, vn, *ident, has_cls)[0],) + attn_bwd_np(qn, kn, vn, don, *ident,
                                                                        has_cls)
    for name, got, ref in zip(("o", "dq", "dk", "dv"), outs[1], refs):
        mx, mean = err_stats(got.double().cpu().numpy(), ref)
        assert mx <= MAX_ABS_TOL and mean <= MEAN_ABS_TOL, (name, mx, mean)
