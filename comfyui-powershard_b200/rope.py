"""RoPE rotation tables in the layout the pre-pass consumes.

The pre-pass applies a per-token table ``freqs[n, D/2, 2, 2]`` (fp32),
i.e. ``freqs[0, :, 0]`` of the reference's ``[1, L, 1, D/2, 2, 2]`` table
(powershard/wan_model.py:325-329).  Inside ComfyUI the table comes from the
model (``WanModel.rope_encode``); these builders produce the same standard
layout for standalone use and for the benchmark:

* ``rope_table_3d`` - Wan video tokens on a (t, h, w) grid, row-major, axes
  split head_dim - 4*(head_dim//6) / 2*(head_dim//6) / 2*(head_dim//6)
  (wan_model.py:1199), pair k of an axis of width d rotated by
  pos * theta^(-2k/d);
* ``rope_table_flux`` - Flux joint attention: text tokens at position 0
  (identity rotation), image tokens at (0, h, w) with axes 16/56/56.
"""
from __future__ import annotations

import torch


def rope_axes(head_dim: int):
    third = head_dim // 6
    return head_dim - 4 * third, 2 * third, 2 * third


def _axis_table(pos: torch.Tensor, width: int, theta: float) -> torch.Tensor:
    k = torch.arange(width // 2, dtype=torch.float64, device=pos.device)
    inv = theta ** (-2.0 * k / width)
    ang = pos.to(torch.float64)[:, None] * inv[None, :]
    cos, sin = torch.cos(ang), torch.sin(ang)
    rot = torch.stack((torch.stack((cos, -sin), -1), torch.stack((sin, cos), -1)), -2)
    return rot.to(torch.float32)                         # [n, width/2, 2, 2]


def rope_table_3d(grid, head_dim: int = 128, theta: float = 10000.0, device=None) -> torch.Tensor:
    """[T*H*W, head_dim/2, 2, 2] fp32 table for a (t, h, w) token grid."""
    t_n, h_n, w_n = grid
    idx = torch.arange(t_n * h_n * w_n, device=device)
    t, h, w = idx // (h_n * w_n), (idx // w_n) % h_n, idx % w_n
    dt, dh, dw = rope_axes(head_dim)
    return torch.cat((_axis_table(t, dt, theta), _axis_table(h, dh, theta), _axis_table(w, dw, theta)), 1)


def rope_table_flux(text_tokens: int, grid_hw, head_dim: int = 128, axes=(16, 56, 56),
                    theta: float = 10000.0, device=None) -> torch.Tensor:
    """[text + H*W, head_dim/2, 2, 2] fp32 table, text first."""
    if sum(axes) != head_dim:
        raise ValueError("Flux axes must sum to head_dim")
    h_n, w_n = grid_hw
    n = text_tokens + h_n * w_n
    pos = torch.zeros(3, n, dtype=torch.int64, device=device)
    img = torch.arange(h_n * w_n, device=device)
    pos[1, text_tokens:] = img // w_n
    pos[2, text_tokens:] = img % w_n
    return torch.cat([_axis_table(pos[i], d, theta) for i, d in enumerate(axes)], 1)
