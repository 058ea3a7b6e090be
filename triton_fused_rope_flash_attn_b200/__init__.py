"""B200-native fused 2D-RoPE FlashAttention (forward + backward).

Drop-in for the public surface of ``fa_rope_full`` (v1kstrand/triton_fused_rope_flash_attn):
``build_axial_rope_pairs``, ``CosSinTable``, ``_sdpa_comp_dtype``,
``TritonAttention`` and ``sdpa_triton_fa_rope``. The compute runs in hand-written
sm_100a CUDA kernels (TMA + tcgen05/TMEM) behind the C ABI of ``include/frsa.h``;
there is no CPU or Triton fallback.
"""
from .rope import build_axial_rope_pairs, CosSinTable  # noqa: F401
from .attention import (  # noqa: F401
    _sdpa_comp_dtype,
    TritonAttention,
    sdpa_triton_fa_rope,
    fused_rope_attention_fwd,
    fused_rope_attention_bwd,
)
from .ops import sdpa_fa_rope_op  # noqa: F401  (registers torch.ops.frsa.*)

__all__ = [
    "build_axial_rope_pairs",
    "CosSinTable",
    "_sdpa_comp_dtype",
    "TritonAttention",
    "sdpa_triton_fa_rope",
    "fused_rope_attention_fwd",
    "fused_rope_attention_bwd",
    "sdpa_fa_rope_op",
]
