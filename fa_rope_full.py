"""Drop-in module name for code written against ``fa_rope_full`` (README usage).

``from fa_rope_full import CosSinTable, sdpa_triton_fa_rope`` resolves to the
B200-native implementation.
"""
from triton_fused_rope_flash_attn_b200 import (  # noqa: F401
    build_axial_rope_pairs,
    CosSinTable,
    _sdpa_comp_dtype,
    TritonAttention,
    sdpa_triton_fa_rope,
)
