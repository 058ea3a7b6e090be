"""The torch.library ops: registration and fake (shape-only) kernels, no GPU needed."""
from __future__ import annotations

import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import triton_fused_rope_flash_attn_b200  # noqa: F401  (registers torch.ops.frsa.*)


def test_ops_registered():
    assert hasattr(torch.ops.frsa, "attn_fwd")
    assert hasattr(torch.ops.frsa, "attn_bwd")


def test_fake_kernels_give_shapes_and_dtypes():
    B, H, N, D = 2, 3, 197, 64
    with FakeTensorMode():
        q, k, v, do = (torch.empty(B, H, N, D, dtype=torch.bfloat16, device="cuda")
                       for _ in range(4))
        cosp = torch.empty(196, D // 2, dtype=torch.float32, device="cuda")
        sinp = torch.empty(196, D // 2, dtype=torch.float32, device="cuda")
        o, lse = torch.ops.frsa.attn_fwd(q, k, v, cosp, sinp, True)
        assert o.shape == (B, H, N, D) and o.dtype == torch.bfloat16
        assert lse.shape == (B, H, N) and lse.dtype == torch.float32
        dq, dk, dv = torch.ops.frsa.attn_bwd(q, k, v, o, lse, do, cosp, sinp, True)
        for g in (dq, dk, dv):
            assert g.shape == (B, H, N, D) and g.dtype == torch.bfloat16
