"""Host-side tables of the Wan 2.2 3D rotary embedding.

The reference builds one complex128 frequency table per head-dim split
(model.py:54-59 `rope_params`, concatenated at :380-384) and, per call,
expands it over the target grid followed by the source grid, padding the rest
of the sequence with ones (model.py:69-95 `rope_apply`, `pad_freqs` :62-66).
Here the table is computed once in float64 with the same formula and handed
to the fused RMSNorm + RoPE kernel as (cos, sin) pairs, together with a
per-token (frame, row, column, rotate) position list.
"""
from __future__ import annotations

import torch


def head_dim_splits(D: int):
    """Pairs of a head given to the frame, row and column axes: the
    reference splits D/2 complex pairs as [c - 2*(c//3), c//3, c//3]
    (model.py:72), i.e. 22 / 21 / 21 for D = 128."""
    c = D // 2
    s1 = c - 2 * (c // 3)
    return s1, s1 + c // 3


def rope_table(D: int, positions: int = 1024, theta: float = 10000.0) -> torch.Tensor:
    """float64 [positions, D/2, 2] (cos, sin): angle = pos / theta**(2i/dim_axis)
    per axis, axes of dims D - 4*(D//6), 2*(D//6), 2*(D//6) (model.py:380-384)."""
    def axis(dim):
        inv = 1.0 / torch.pow(torch.tensor(theta, dtype=torch.float64),
                              torch.arange(0, dim, 2, dtype=torch.float64).div(dim))
        return torch.outer(torch.arange(positions, dtype=torch.float64), inv)
    ang = torch.cat([axis(D - 4 * (D // 6)), axis(2 * (D // 6)), axis(2 * (D // 6))], dim=1)
    assert ang.shape[1] == D // 2
    # torch.polar on the CPU, as the reference builds it: its cos / sin can
    # differ from torch.cos / torch.sin in the last bit
    return torch.view_as_real(torch.polar(torch.ones_like(ang), ang)).contiguous()


def grid_positions(grid) -> torch.Tensor:
    """int32 [f*h*w, 4]: (frame, row, column, 1) in the reference's token order
    (row-major over f, h, w, the order of `flatten(2)` in model.py:422-423)."""
    f, h, w = grid
    ff, hh, ww = torch.meshgrid(torch.arange(f), torch.arange(h), torch.arange(w), indexing="ij")
    return torch.stack([ff.reshape(-1), hh.reshape(-1), ww.reshape(-1), torch.ones(f * h * w, dtype=torch.long)],
                       dim=1).to(torch.int32)


def token_positions(target_grid, source_grid, seq_len: int) -> torch.Tensor:
    """int32 [seq_len, 4] for the joint sequence [target | source | padding]:
    padding tokens get rotate = 0 (the reference multiplies them by ones)."""
    t = grid_positions(target_grid)
    s = grid_positions(source_grid)
    n = t.shape[0] + s.shape[0]
    if n > seq_len:
        raise ValueError(f"{n} video tokens exceed seq_len={seq_len}")
    pad = torch.zeros(seq_len - n, 4, dtype=torch.int32)
    return torch.cat([t, s, pad]).contiguous()
