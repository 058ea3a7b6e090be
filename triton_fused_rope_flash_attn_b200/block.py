"""The caller of the path: a ViT self-attention block with fused 2D RoPE.

The reference's README benchmarks its kernel inside timm's RoPE ViT blocks
(README.md:156-159): ``x -> qkv = Linear(x) -> split heads -> fused RoPE SDPA
-> merge heads -> Linear``. timm is not a dependency here, so this is a
self-contained block with the same structure, for use in models and for
timing a whole attention layer. The projections are plain ``nn.Linear``
(cuBLAS); the attention is this package's kernel.
"""
from __future__ import annotations

import torch
from torch import nn

from . import qkv as _qkv
from .attention import sdpa_triton_fa_rope
from .rope import CosSinTable


class RopeAttention(nn.Module):
    """Multi-head self-attention over a CLS + ``H_img x H_img`` patch grid with
    2D axial RoPE applied to queries and keys inside the attention kernel.

    Input and output: ``[B, N, dim]`` with ``N = H_img**2 + has_cls``.
    """

    def __init__(self, dim: int, num_heads: int, H_img: int = 14, has_cls: bool = True,
                 rope_base: float = 100.0, qkv_bias: bool = True, device=None, dtype=None,
                 fused_qkv: bool = False):
        super().__init__()
        assert dim % num_heads == 0, "dim must be divisible by num_heads"
        self.num_heads = num_heads
        self.head_dim = dim // num_heads
        self.H_img = H_img
        self.has_cls = has_cls
        self.qkv = nn.Linear(dim, 3 * dim, bias=qkv_bias, device=device, dtype=dtype)
        self.proj = nn.Linear(dim, dim, device=device, dtype=dtype)
        dev = device if device is not None else "cuda"
        self.rope = CosSinTable(rope_base, H_img, self.head_dim, device=dev)
        # fused_qkv: the projection kernel applies the RoPE in its epilogue and
        # the attention rotates nothing (rope=False).
        self.fused_qkv = fused_qkv

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        B, N, C = x.shape
        if self.fused_qkv and _qkv.supported(C, self.num_heads, x.dtype):
            q, k, v = _qkv.qkv_rope(x, self.qkv.weight, self.qkv.bias, self.rope, self.num_heads,
                                    self.has_cls)
            o = sdpa_triton_fa_rope(q, k, v, None, has_cls=self.has_cls, H_img=self.H_img,
                                    rope=False)
            return self.proj(o.transpose(1, 2).reshape(B, N, C))
        qkv = self.qkv(x).view(B, N, 3, self.num_heads, self.head_dim)
        q, k, v = qkv.permute(2, 0, 3, 1, 4).unbind(0)        # [B, H, N, D] views
        o = sdpa_triton_fa_rope(q, k, v, self.rope, has_cls=self.has_cls, H_img=self.H_img)
        return self.proj(o.transpose(1, 2).reshape(B, N, C))
