"""GPU: the torch.library ops give the same results as the autograd.Function
path (same kernels), pass torch's op checks, and trace under torch.compile
without a graph break."""
from __future__ import annotations

import pytest
import torch

from tests.helpers import seeded_inputs

pytestmark = pytest.mark.gpu


def _inputs(dtype=torch.bfloat16, B=2, H=3, side=14, has_cls=True, D=64):
    from triton_fused_rope_flash_attn_b200 import CosSinTable
    N = side * side + (1 if has_cls else 0)
    q, k, v, do = (t.to("cuda", dtype) for t in seeded_inputs(B, H, N, D, 1.0, 5))
    return q, k, v, do, CosSinTable(100.0, side, D, device="cuda")


def _fwd_bwd(fn, q, k, v, do, cs):
    q, k, v = (t.clone().requires_grad_(True) for t in (q, k, v))
    o = fn(q, k, v, cs)
    o.backward(do)
    return o.detach(), q.grad, k.grad, v.grad


def test_op_matches_autograd_function():
    from triton_fused_rope_flash_attn_b200 import sdpa_fa_rope_op, sdpa_triton_fa_rope
    q, k, v, do, cs = _inputs()
    a = _fwd_bwd(sdpa_triton_fa_rope, q, k, v, do, cs)
    b = _fwd_bwd(sdpa_fa_rope_op, q, k, v, do, cs)
    for x, y in zip(a, b):
        assert torch.equal(x, y)


def test_op_under_autocast_fp32_inputs():
    from triton_fused_rope_flash_attn_b200 import sdpa_fa_rope_op, sdpa_triton_fa_rope
    q, k, v, do, cs = _inputs(dtype=torch.float32)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        a = _fwd_bwd(sdpa_triton_fa_rope, q, k, v, do, cs)
        b = _fwd_bwd(sdpa_fa_rope_op, q, k, v, do, cs)
    assert a[0].dtype == torch.float32 and b[0].dtype == torch.float32
    for x, y in zip(a, b):
        assert torch.equal(x, y)


def test_compile_fullgraph():
    from triton_fused_rope_flash_attn_b200 import sdpa_fa_rope_op
    q, k, v, do, cs = _inputs()

    def f(q, k, v):
        return sdpa_fa_rope_op(q, k, v, cs) * 2.0

    compiled = torch.compile(f, fullgraph=True, backend="aot_eager")
    a = _fwd_bwd(lambda q, k, v, cs: f(q, k, v), q, k, v, do, cs)
    b = _fwd_bwd(lambda q, k, v, cs: compiled(q, k, v), q, k, v, do, cs)
    for x, y in zip(a, b):
        assert torch.equal(x, y)


def test_opcheck():
    q, k, v, do, cs = _inputs(B=1, H=2, side=5)
    args = (q, k, v, cs.COSP, cs.SINP, True)
    torch.library.opcheck(torch.ops.frsa.attn_fwd.default, args,
                          test_utils=("test_schema", "test_faketensor", "test_autograd_registration"))
