"""GPU parity against the reference's own Triton kernels, run on the same B200.

The reference module (fa_rope_full .py, an untracked copy in ``baseline/_ref``)
is imported by path and called through its public autograd class
``TritonAttention.apply(Q, K, V, cos_sin, H_img, has_cls)``
(fa_rope_full .py:1011-1138). Both arms get identical seeded bf16 inputs at
the full ViT-S, ViT-B and ViT-L attention shapes. Asserted, per tensor
(O, dQ, dK, dV):

  * this repository's outputs against an fp32 torch evaluation of the same
    operation (PyTorch SDPA over Python-rotated q, k, the harness the
    reference's README.md:123-136 describes): max abs <= 3e-2, mean <= 1e-3;
  * this repository's outputs against the reference kernel's outputs: the
    same bar, with the max bound widened by the reference's own max error
    against the fp32 evaluation (the reference publishes a dK max error of
    3.1e-2 itself, README.md:130-133, so its own outputs can sit outside a
    3e-2 ball around the exact result).

Both arms' errors against the fp32 evaluation are printed (``pytest -s``). At
ViT-H (D = 80) the reference cannot compile (``tl.arange`` over a head dim
that is not a power of two): the test records that failure.
"""
from __future__ import annotations

import pytest
import torch

from bench import load_reference_triton
from tests.test_gpu_fullsize import _reference

pytestmark = pytest.mark.gpu

SHAPES = {"vit_s": (512, 6, 14, True, 64), "vit_b": (256, 12, 14, True, 64),
          "vit_l": (128, 16, 24, False, 64)}


def _ref_module():
    mod, why = load_reference_triton()
    if mod is None:
        pytest.skip(why)
    return mod


def _inputs(B, H, N, D, seed=11):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return [torch.randn(B, H, N, D, device="cuda", generator=g).bfloat16() for _ in range(4)]


@pytest.mark.parametrize("name", sorted(SHAPES))
def test_matches_reference_triton(name):
    ref = _ref_module()
    from triton_fused_rope_flash_attn_b200 import CosSinTable, _lib, sdpa_triton_fa_rope
    B, H, side, has_cls, D = SHAPES[name]
    N = side * side + int(has_cls)
    q, k, v, do = _inputs(B, H, N, D)

    # Reference arm (its own table module and kernels).
    cs_ref = ref.CosSinTable(100.0, side, D, device="cuda")
    qr, kr, vr = (t.clone().requires_grad_(True) for t in (q, k, v))
    o_ref = ref.TritonAttention.apply(qr, kr, vr, cs_ref, side, has_cls)
    o_ref.backward(do)
    ref_out = (o_ref.detach(), qr.grad, kr.grad, vr.grad)

    # This repository's arm through its drop-in entry point.
    cs = CosSinTable(100.0, side, D, device="cuda")
    assert torch.equal(cs.COSP, cs_ref.COSP) and torch.equal(cs.SINP, cs_ref.SINP)
    qo, ko, vo = (t.clone().requires_grad_(True) for t in (q, k, v))
    o = sdpa_triton_fa_rope(qo, ko, vo, cs, has_cls=has_cls, H_img=side)
    o.backward(do)
    our_out = (o.detach(), qo.grad, ko.grad, vo.grad)
    torch.cuda.synchronize()
    assert _lib.load().frsa_query_status() == 0

    exact = _reference(q, k, v, do, cs.COSP, cs.SINP, has_cls)
    for tname, ours, theirs, ex in zip(("O", "dQ", "dK", "dV"), our_out, ref_out, exact):
        e_ours = (ours.float() - ex).abs()
        e_ref = (theirs.float() - ex).abs()
        d = (ours.float() - theirs.float()).abs()
        print(f"[{name} {tname}] ours-vs-fp32 max {float(e_ours.max()):.3e} mean "
              f"{float(e_ours.mean()):.3e} | reference-vs-fp32 max {float(e_ref.max()):.3e} "
              f"mean {float(e_ref.mean()):.3e} | ours-vs-reference max {float(d.max()):.3e} "
              f"mean {float(d.mean()):.3e}")
        assert float(e_ours.max()) <= 3e-2 and float(e_ours.mean()) <= 1e-3, tname
        assert float(d.max()) <= 3e-2 + float(e_ref.max()), tname
        assert float(d.mean()) <= 1e-3, tname


def test_reference_triton_rejects_head_dim_80():
    """ViT-H's D = 80: the reference's kernels do not compile (a power-of-two
    ``tl.arange`` over HEAD_DIM), so there is no reference number there."""
    ref = _ref_module()
    q, k, v, do = _inputs(1, 2, 37 * 37 + 1, 80)
    cs_ref = ref.CosSinTable(100.0, 37, 80, device="cuda")
    with pytest.raises(Exception):
        o = ref.TritonAttention.apply(q, k, v, cs_ref, 37, True)
        torch.cuda.synchronize()
        del o
