"""Tile bitmaps and MMA occupancy counts restated with numpy (test oracle).

Bitmap layout (include/spmlp.h): bit (g % 32) of word [r * words + g // 32] is
set iff the 16-token x 64-feature tile (r, g) of h holds a nonzero value;
words = ceil(ceil(F / 64) / 32).  A tile's bit is the OR of the reference
gate's element mask ``gate(z) != 0`` over the tile.
"""
from __future__ import annotations

import numpy as np
import torch

ROWS, COLS = 16, 64


def words_per_group(features: int, cols: int = COLS) -> int:
    return (-(-features // cols) + 31) // 32


def tile_mask(h: torch.Tensor | np.ndarray, rows: int = ROWS, cols: int = COLS) -> np.ndarray:
    """Boolean [ceil(T/rows), ceil(F/cols)]: tile holds a nonzero (-0.0 counts as zero)."""
    a = h.detach().cpu().float().numpy() if isinstance(h, torch.Tensor) else np.asarray(h, dtype=np.float32)
    t, f = a.shape
    tr, tc = -(-t // rows), -(-f // cols)
    pad = np.zeros((tr * rows, tc * cols), dtype=bool)
    pad[:t, :f] = a != 0
    return pad.reshape(tr, rows, tc, cols).any(axis=(1, 3))


def pack_bits(mask: np.ndarray) -> np.ndarray:
    """Pack a boolean [groups, tiles] mask into uint32 words (LSB = lowest tile)."""
    groups, tiles = mask.shape
    words = (tiles + 31) // 32
    padded = np.zeros((groups, words * 32), dtype=np.uint64)
    padded[:, :tiles] = mask
    shifts = np.arange(32, dtype=np.uint64)
    return (padded.reshape(groups, words, 32) << shifts).sum(axis=2).astype(np.uint32)


def unpack_bits(words: np.ndarray, tiles: int) -> np.ndarray:
    w = np.asarray(words, dtype=np.uint32)
    bits = (w[..., None] >> np.arange(32, dtype=np.uint32)) & 1
    return bits.reshape(w.shape[0], -1)[:, :tiles].astype(bool)


def tile_bits(h, rows: int = ROWS, cols: int = COLS) -> np.ndarray:
    """Packed bitmap of h, flattened to the kernel's 1-D word order."""
    return pack_bits(tile_mask(h, rows, cols)).reshape(-1)


def skip_counts(mask: np.ndarray, k_features: int, n_tiles: int, m_tile: int = 128, row_group: int = ROWS,
                granule: int = COLS) -> tuple[int, int]:
    """Issued / skipped K16 MMA steps of the sparse down-projection.

    mask: boolean [row_groups, k_granules] (16-token groups x ``granule``-wide K
    groups).  A 128-token tile issues the K16 steps of every granule live in any
    of its row groups; each tile is repeated for each of the ``n_tiles`` output
    column tiles.  Restates the issued/bypassed split of
    runs/042-2026-09-20-pythia70m-sparse-scale/tile_oracle.py:4-20 for our tile shape.
    """
    groups_per_tile = m_tile // row_group
    g = mask.shape[0]
    pad = -(-g // groups_per_tile) * groups_per_tile
    m = np.zeros((pad, mask.shape[1]), dtype=bool)
    m[:g] = mask
    live = m.reshape(-1, groups_per_tile, mask.shape[1]).any(axis=1)
    steps_per_granule = granule // 16
    issued = int(live.sum()) * steps_per_granule * n_tiles
    total = live.shape[0] * (k_features // 16) * n_tiles
    return issued, total - issued


def reference_counts(value: torch.Tensor, rows: int, skip: bool = True, max_short: int = 2, n_out: int = 512,
                     fast_weights: bool = True) -> list[int]:
    """The reference's M8/M16 x K16 accounting (runs/042-2026-09-20-pythia70m-sparse-scale/tile_oracle.py:4-20).

    Returns [issued, bypassed, scalar] where issued/bypassed count m16n8k16 MMAs
    over n_out output columns and scalar counts products done by the short-row
    SIMT path (rows with <= max_short nonzeros).
    """
    flat = value.reshape(-1, value.shape[-1])
    if rows not in (8, 16) or flat.shape[0] % rows or flat.shape[1] % 16:
        raise ValueError("rows must be 8 or 16 and shapes aligned")
    groups, ktiles = flat.shape[0] // rows, flat.shape[1] // 16
    potential = groups * ktiles * (n_out // 8)
    if not skip:
        return [potential, 0, 0]
    nonzero = flat != 0
    nnz = nonzero.sum(-1)
    safe = ((flat == 0) | ((flat.abs() >= 2.0 ** -50) & (flat.abs() <= 2.0 ** 50))).all(-1)
    short = (nnz <= max_short) & safe & fast_weights
    active = nonzero & ~short[:, None]
    active_tiles = active.reshape(groups, rows, ktiles, 16).any(1).any(-1).sum()
    issued = int(active_tiles) * (n_out // 8)
    scalar = int(nnz[short].sum()) * n_out
    return [issued, potential - issued, scalar]
