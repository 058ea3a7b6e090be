"""2D axial RoPE pair tables (fa_rope_full .py:10-63, 1140-1166).

The tables are built with the same float32 torch operations as the reference,
on the requested device, so they agree with the reference bit for bit on the
same device: ``inv_freq[k] = base ** (-k / P)`` with ``P = D/4``; the 1-D angle
``pos * inv_freq`` for ``pos < side``; pair column ``k < P`` uses the row index
``lin // side`` of the flattened position and pair column ``P + k`` uses the
column index ``lin % side``.
"""
from __future__ import annotations

import torch


def build_axial_rope_pairs(side_len: int, head_dim: int, device: torch.device,
                           base: float = 10000.0):
    """Return ``(cos_pairs, sin_pairs)``, float32 contiguous ``[side_len**2, head_dim//2]``."""
    assert head_dim % 4 == 0, "need head_dim divisible by 4 for 2D axial RoPE"
    per_axis = head_dim // 4
    k = torch.arange(0, per_axis, device=device)
    inv_freq = base ** (-k / per_axis)                     # float32 [P]
    coord = torch.arange(side_len, device=device)
    ang = torch.outer(coord, inv_freq)                     # float32 [side, P]
    cos1, sin1 = torch.cos(ang), torch.sin(ang)
    lin = torch.arange(side_len * side_len, device=device)
    row, col = lin // side_len, lin % side_len
    cos_pairs = torch.cat((cos1[row], cos1[col]), dim=1).contiguous()
    sin_pairs = torch.cat((sin1[row], sin1[col]), dim=1).contiguous()
    return cos_pairs, sin_pairs


class CosSinTable(torch.nn.Module):
    """Pairwise axial RoPE tables for an ``H_img x H_img`` grid.

    Buffers ``COSP`` and ``SINP`` are float32 ``[H_img**2, D//2]``; the names
    match the reference so existing ``state_dict``s load unchanged.
    """

    def __init__(self, base: float, H_img: int = 14, D: int = 64, device: str = "cuda"):
        super().__init__()
        cos_pairs, sin_pairs = build_axial_rope_pairs(H_img, D, torch.device(device), base)
        self.register_buffer("COSP", cos_pairs)
        self.register_buffer("SINP", sin_pairs)

    def tables(self):
        """``(COSP, SINP)``, each ``[N_pos, D2]`` float32."""
        return self.COSP, self.SINP
