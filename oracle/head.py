"""Vocabulary-head oracle (test infrastructure; see oracle/__init__.py).

Reference: runs/068-2026-10-08-pythia14m-aligned-vocabulary-tiles/inference/head.cu:9-16
(prepare: fp32 corner certificate per 16-row group, then fp16 cast),
head.cu:18-77 (project: K16 groups whose certificate failed are skipped, every
vocabulary logit is written) and head.py:31-37 (weight fragment packing).
"""
from __future__ import annotations

import numpy as np
import torch

from . import bitmap, gates


def support_mask(x: torch.Tensor, kappa: float) -> np.ndarray:
    """Boolean [ceil(T/16), d/16]: fp32 corner x[16r, 16j] > kappa (head.cu:12)."""
    x = x.float()
    corners = x[::16, ::16]
    return (corners > float(np.float32(kappa))).numpy()


def support_bits(x: torch.Tensor, kappa: float) -> np.ndarray:
    return bitmap.pack_bits(support_mask(x, kappa)).reshape(-1)


def prepare(x: torch.Tensor, kappa: float, dtype: torch.dtype) -> tuple[torch.Tensor, np.ndarray]:
    """Gated head input in ``dtype`` (dead 16x16 tiles zeroed) and its support bits."""
    gated = gates.corner(x.float(), float(np.float32(kappa)), 16, 16)
    return gated.to(dtype), support_bits(x, kappa)


def logits(x: torch.Tensor, w: torch.Tensor, dtype: torch.dtype | None = None,
           acc: torch.dtype = torch.float32) -> torch.Tensor:
    """x w^T with fp32 (or fp64) accumulation, optionally rounded once to dtype."""
    out = x.to(acc) @ w.to(acc).T
    return out if dtype is None else out.to(dtype)


def pack_weight(weight: torch.Tensor) -> torch.Tensor:
    """head.py:31-37 pack_weight: exact fragment permutation of a [V, 128] weight."""
    vocabulary, width = weight.shape
    if width != 128:
        raise ValueError("D128 weights required")
    padded = torch.nn.functional.pad(weight, (0, 0, 0, (-vocabulary) % 8))
    return padded.reshape(-1, 8, 8, 2, 8).permute(2, 0, 3, 1, 4).contiguous().reshape(8, -1, 128)


def unpack_weight(packed: torch.Tensor) -> torch.Tensor:
    return packed.reshape(8, -1, 2, 8, 8).permute(1, 3, 0, 2, 4).reshape(-1, 128)

