"""CPU oracle for the fused 2D-RoPE SDPA path (TEST INFRASTRUCTURE ONLY).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this package, and only as the checker or the timed CPU
baseline. The product path (``triton_fused_rope_flash_attn_b200``) never
imports it and has no CPU fallback.
"""
from .frsa_oracle import (  # noqa: F401
    rope_tables_np,
    rotate_pairs_np,
    unrotate_pairs_np,
    attn_fwd_np,
    attn_bwd_np,
    attn_fwd_bwd_torch,
    flops_fwd_bwd,
)
