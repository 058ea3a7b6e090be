"""The CPU oracle pinned against the golden fixtures made from the reference.

``tests/golden/tables.npz`` holds the reference's own ``build_axial_rope_pairs``
output; ``tests/golden/attn_cases.npz`` holds seeded small cases evaluated by
the reference's described correctness harness (PyTorch SDPA + Python 2D RoPE)
in float64 on the reference's tables (tests/golden/make_golden.py).
"""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from oracle import (attn_bwd_np, attn_fwd_bwd_torch, attn_fwd_np, rope_tables_np,
                    rotate_pairs_np, unrotate_pairs_np)

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _tables():
    return np.load(os.path.join(GOLD, "tables.npz"))


def _cases():
    z = np.load(os.path.join(GOLD, "attn_cases.npz"))
    out = []
    for i in range(int(z["n_cases"])):
        B, H, side, has_cls, D, base, amp = z[f"c{i}_meta"]
        out.append(dict(has_cls=bool(has_cls), **{n: z[f"c{i}_{n}"] for n in
                                                  ("q", "k", "v", "do", "cos", "sin", "o", "dq",
                                                   "dk", "dv")}))
    return out


@pytest.mark.parametrize("key", sorted({k[4:] for k in _tables().files}))
def test_oracle_tables_match_reference(key):
    side, D, base = (int(x) for x in key.split("_"))
    t = _tables()
    c, s = rope_tables_np(side, D, float(base))
    # numpy's float32 cos/pow may differ from torch's by a few ulp
    np.testing.assert_allclose(c, t["cos_" + key], atol=4e-6, rtol=0)
    np.testing.assert_allclose(s, t["sin_" + key], atol=4e-6, rtol=0)


@pytest.mark.parametrize("key", sorted({k[4:] for k in _tables().files}))
def test_product_tables_bitwise_equal_reference(key):
    """The package's table builder reproduces the reference bit for bit (CPU)."""
    from triton_fused_rope_flash_attn_b200 import CosSinTable, build_axial_rope_pairs
    side, D, base = (int(x) for x in key.split("_"))
    t = _tables()
    c, s = build_axial_rope_pairs(side, D, torch.device("cpu"), float(base))
    assert c.dtype == torch.float32 and c.is_contiguous() and c.shape == (side * side, D // 2)
    assert np.array_equal(c.numpy(), t["cos_" + key])
    assert np.array_equal(s.numpy(), t["sin_" + key])
    m = CosSinTable(float(base), side, D, device="cpu")
    assert set(m.state_dict()) == {"COSP", "SINP"}
    assert np.array_equal(m.tables()[0].numpy(), t["cos_" + key])


@pytest.mark.parametrize("idx", range(7))
def test_oracle_attention_matches_golden(idx):
    c = _cases()[idx]
    q, k, v, do = (c[n].astype(np.float64) for n in ("q", "k", "v", "do"))
    o, _ = attn_fwd_np(q, k, v, c["cos"], c["sin"], c["has_cls"])
    dq, dk, dv = attn_bwd_np(q, k, v, do, c["cos"], c["sin"], c["has_cls"])
    for got, name in ((o, "o"), (dq, "dq"), (dk, "dk"), (dv, "dv")):
        np.testing.assert_allclose(got, c[name], atol=1e-10, rtol=1e-9, err_msg=name)


def test_torch_harness_matches_golden():
    c = _cases()[6]  # N=197
    q, k, v, do = (torch.from_numpy(c[n]).double() for n in ("q", "k", "v", "do"))
    o, dq, dk, dv = attn_fwd_bwd_torch(q, k, v, do, c["cos"], c["sin"], c["has_cls"])
    for got, name in ((o, "o"), (dq, "dq"), (dk, "dk"), (dv, "dv")):
        np.testing.assert_allclose(got.numpy(), c[name], atol=1e-10, err_msg=name)


def test_single_key_output_is_v():
    """N = 1: softmax over one key is 1, so O = V and dQ = dK = 0, dV = dO."""
    cos, sin = rope_tables_np(1, 64, 100.0)
    rng = np.random.default_rng(0)
    q, k, v, do = (rng.standard_normal((1, 2, 1, 64)) for _ in range(4))
    o, lse = attn_fwd_np(q, k, v, cos, sin, False)
    np.testing.assert_allclose(o, v, atol=1e-12)
    dq, dk, dv = attn_bwd_np(q, k, v, do, cos, sin, False)
    np.testing.assert_allclose(dq, 0, atol=1e-12)
    np.testing.assert_allclose(dk, 0, atol=1e-12)
    np.testing.assert_allclose(dv, do, atol=1e-12)


def test_rotation_is_orthogonal_and_cls_identity():
    cos, sin = rope_tables_np(3, 16, 100.0)
    rng = np.random.default_rng(1)
    x = rng.standard_normal((2, 10, 16))
    r = rotate_pairs_np(x, cos, sin, True)
    np.testing.assert_allclose(unrotate_pairs_np(r, cos, sin, True), x, atol=1e-12)
    np.testing.assert_allclose(r[:, 0], x[:, 0])                    # CLS untouched
    np.testing.assert_allclose(np.linalg.norm(r, axis=-1), np.linalg.norm(x, axis=-1))
    # table row 0 has angle 0 everywhere -> token 1 (first patch) is untouched too
    np.testing.assert_allclose(r[:, 1], x[:, 1], atol=1e-12)


def test_table_axis_convention():
    """Pair columns < D/4 follow the row index lin // side, the rest lin % side."""
    cos, _ = rope_tables_np(14, 64, 100.0)
    assert cos[1, 0] == 1.0 and cos[14, 0] != 1.0        # lin 14 = row 1
    assert cos[1, 16] != 1.0 and cos[14, 16] == 1.0      # lin 1 = col 1
