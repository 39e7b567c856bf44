"""Interleaved rotary position embedding.

Parity: astrai/model/components/rope.py. Angles ``pos * base^(-2i/d)`` are
computed in float64 and stored as fp32 (cos, sin) pairs; pairs (x[2i],
x[2i+1]) are rotated. NTK scaling changes the base to
``base * factor^(d/(d-2))``.

On CUDA the rotation runs in place on the q / k column ranges of the fused
QKV projection output, so q and k are never copied.
"""

from __future__ import annotations

from typing import Optional

import torch

from astrai_b200.ops._ext import native


def ntk_base(base: float, dim: int, factor: float) -> float:
    return base * (factor ** (dim / (dim - 2)))


def rope_table(dim: int, max_len: int, base: float = 10000.0, device=None) -> torch.Tensor:
    """fp32 ``[max_len, dim/2, 2]`` table of (cos, sin)."""
    inv = base ** (-torch.arange(0, dim, 2, dtype=torch.float64, device=device) / dim)
    ang = torch.outer(torch.arange(max_len, dtype=torch.float64, device=device), inv).float()
    return torch.stack([torch.cos(ang), torch.sin(ang)], dim=-1).contiguous()


def apply_rope_reference(x: torch.Tensor, cs: torch.Tensor) -> torch.Tensor:
    """x: [B, S, H, D]; cs: [B, S, D/2, 2] (already indexed by position)."""
    xf = x.float().reshape(*x.shape[:-1], -1, 2)
    c = cs[..., 0].unsqueeze(2)
    s = cs[..., 1].unsqueeze(2)
    x0, x1 = xf[..., 0], xf[..., 1]
    out = torch.stack([x0 * c - x1 * s, x0 * s + x1 * c], dim=-1)
    return out.flatten(-2).to(x.dtype)


def rope_inplace(buf: torch.Tensor, col0: int, n_heads: int, head_dim: int, table: torch.Tensor,
                 positions: Optional[torch.Tensor], seq_len: int, inverse: bool = False,
                 rot_dim: Optional[int] = None, rot_off: int = 0) -> None:
    """Rotate heads stored in ``buf[:, col0 : col0 + n_heads*head_dim]`` in place (CUDA).

    ``positions`` is an int32 tensor with one entry per row of ``buf`` or None
    (then row ``r`` has position ``r % seq_len``). ``rot_dim``/``rot_off``
    restrict the rotation to a slice of each head (MLA rope part).
    """
    rd = head_dim if rot_dim is None else rot_dim
    native().rope_(buf, col0, n_heads, head_dim, positions, seq_len, table, inverse, rd, rot_off)
