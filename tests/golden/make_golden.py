"""Generate the golden fixtures under tests/golden/ from the reference itself.

Run in a container where the reference checkout is present:

    python tests/golden/make_golden.py /path/to/reference

What it writes (all small ``.npz`` files):

* ``tables.npz`` — ``build_axial_rope_pairs`` outputs of the reference
  (fa_rope_full .py:10-63), run on CPU, for several ``(H_img, D, base)``.
* ``attn_cases.npz`` — seeded small attention cases: fp32 inputs, the
  reference's tables, and the outputs of the reference's described
  correctness harness (PyTorch SDPA + Python 2D RoPE, README.md:123-136)
  evaluated in float64 with torch autograd: ``o, dq, dk, dv``.

The reference's Triton kernels need a GPU and are not run here; the attention
fixtures pin the oracle to an independent (autograd) evaluation of the same
math on the reference's own tables.
"""
from __future__ import annotations

import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

TABLE_CASES = [(14, 64, 100.0), (24, 64, 100.0), (37, 80, 100.0), (2, 4, 10000.0),
               (3, 8, 10000.0), (1, 64, 100.0), (7, 80, 10000.0)]

# (B, H, H_img, has_cls, D, base, input scale)
ATTN_CASES = [
    (1, 2, 1, True, 64, 100.0, 1.0),     # N=2
    (1, 1, 1, False, 64, 100.0, 1.0),    # N=1
    (1, 2, 2, True, 64, 100.0, 1.0),     # N=5
    (2, 1, 3, False, 64, 100.0, 1.0),    # N=9
    (1, 2, 5, True, 64, 100.0, 1.0),     # N=26
    (1, 1, 7, False, 80, 100.0, 2.0),    # N=49, D=80
    (1, 1, 14, True, 64, 100.0, 1.0),    # N=197
]


def load_reference(ref_dir: str):
    path = os.path.join(ref_dir, "fa_rope_full .py")
    spec = importlib.util.spec_from_file_location("fa_rope_full_reference", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def harness_fp64(q, k, v, do, cos, sin, has_cls):
    """PyTorch SDPA over Python-rotated q, k in float64 (README.md:123-136)."""
    import torch.nn.functional as F
    N = q.shape[-2]
    off = 1 if has_cls else 0
    C = torch.ones(N, cos.shape[1], dtype=torch.float64)
    S = torch.zeros(N, cos.shape[1], dtype=torch.float64)
    C[off:] = cos[: N - off].double()
    S[off:] = sin[: N - off].double()

    def rot(x):
        e, o = x[..., 0::2], x[..., 1::2]
        return torch.stack((e * C - o * S, o * C + e * S), dim=-1).flatten(-2)

    q, k, v = (t.double().requires_grad_(True) for t in (q, k, v))
    o = F.scaled_dot_product_attention(rot(q), rot(k), v)
    o.backward(do.double())
    return o.detach(), q.grad, k.grad, v.grad


def main(ref_dir: str):
    ref = load_reference(ref_dir)
    tabs = {}
    for side, D, base in TABLE_CASES:
        c, s = ref.build_axial_rope_pairs(side, D, torch.device("cpu"), base)
        key = f"{side}_{D}_{int(base)}"
        tabs[f"cos_{key}"] = c.numpy()
        tabs[f"sin_{key}"] = s.numpy()
    np.savez_compressed(os.path.join(HERE, "tables.npz"), **tabs)

    out = {}
    for idx, (B, H, side, has_cls, D, base, amp) in enumerate(ATTN_CASES):
        N = side * side + (1 if has_cls else 0)
        g = torch.Generator().manual_seed(1000 + idx)
        q = torch.randn(B, H, N, D, generator=g) * amp
        k = torch.randn(B, H, N, D, generator=g) * amp
        v = torch.randn(B, H, N, D, generator=g) * amp
        do = torch.randn(B, H, N, D, generator=g)
        cos, sin = ref.build_axial_rope_pairs(side, D, torch.device("cpu"), base)
        o, dq, dk, dv = harness_fp64(q, k, v, do, cos, sin, has_cls)
        meta = np.array([B, H, side, int(has_cls), D, base, amp], dtype=np.float64)
        for name, t in (("q", q), ("k", k), ("v", v), ("do", do), ("cos", cos), ("sin", sin)):
            out[f"c{idx}_{name}"] = t.numpy().astype(np.float32)
        for name, t in (("o", o), ("dq", dq), ("dk", dk), ("dv", dv)):
            out[f"c{idx}_{name}"] = t.numpy()
        out[f"c{idx}_meta"] = meta
    out["n_cases"] = np.array(len(ATTN_CASES))
    np.savez_compressed(os.path.join(HERE, "attn_cases.npz"), **out)
    print("wrote", os.path.join(HERE, "tables.npz"), os.path.join(HERE, "attn_cases.npz"))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <reference checkout dir>")
    main(sys.argv[1])
