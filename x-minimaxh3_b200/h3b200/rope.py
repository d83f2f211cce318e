"""RoPE rotation tables for the packed (t, h, w) token grid.

The table is an input of the norm-RoPE kernel, built once per DiT call as in
the reference (h3serve/native_engine/model/dit.py:669-671): per-axis angles
``pos * inv_freq`` concatenated (layers.py:51-58, here with a per-axis
frequency width such as 44/42/42 head dims), packed as ``[[cos, -sin],
[sin, cos]]`` (layers.py:61-69). cos/sin are evaluated in float64 and rounded
to fp32.
"""

from __future__ import annotations

import torch


def rope_axis_inv_freq(dim: int, base: float = 10000.0, device=None) -> torch.Tensor:
    """``1 / base^(arange(0, dim, 2) / dim)`` for one axis of ``dim`` head dims, evaluated in
    float64 and rounded to fp32."""
    e = torch.arange(0, dim, 2, dtype=torch.float64, device=device) / dim
    return (1.0 / (base ** e)).to(torch.float32)


def rope_grid_table(grid, dims=(44, 42, 42), base: float = 10000.0, token_slice=None, device="cuda") -> torch.Tensor:
    """fp32 [M, sum(dims)/2, 2, 2] rotation table for a row-major (t, h, w) grid.

    ``token_slice=(lo, hi)`` builds the rows of a contiguous token shard."""
    t, h, w = grid
    m = t * h * w
    lo, hi = (0, m) if token_slice is None else token_slice
    idx = torch.arange(lo, hi, dtype=torch.int64, device=device)
    pos = torch.stack([idx // (h * w), (idx // w) % h, idx % w], dim=1).to(torch.float32)
    ang = torch.cat([pos[:, a:a + 1] * rope_axis_inv_freq(d, base, device).reshape(1, -1)
                     for a, d in enumerate(dims)], dim=1)
    a64 = ang.to(torch.float64)
    c = torch.cos(a64).to(torch.float32)
    s = torch.sin(a64).to(torch.float32)
    return torch.stack([c, -s, s, c], dim=-1).reshape(hi - lo, ang.shape[1], 2, 2).contiguous()
