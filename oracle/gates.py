"""Gate operators restated on the CPU (test oracle; see oracle/__init__.py)."""
from __future__ import annotations

import math

import numpy as np
import torch


def round_kappa(kappa: float, dtype: torch.dtype) -> float:
    """kappa as the activation dtype sees it.

    Reference: runs/063-2026-10-07-pythia14m-tile-specialized-kernel/kernel.py:17-19 —
    TensorIterator converts the wrapped Python scalar to the tensor's dtype before
    the comparison, i.e. float(torch.tensor(kappa, dtype=dtype)).
    """
    return float(torch.tensor(kappa, dtype=dtype))


def one_sided(z: torch.Tensor, kappa: float) -> torch.Tensor:
    """sites.py:86-94 FixedOneSidedThreshold: keep z >= kappa (equality survives)."""
    return z.masked_fill(z < kappa, 0.0)


def symmetric(z: torch.Tensor, kappa: float) -> torch.Tensor:
    """sites.py:97-107 FixedSymmetricThreshold: keep |z| >= kappa; kappa == 0 is the identity."""
    if kappa == 0.0:
        return z
    return z.masked_fill(z.abs() < kappa, 0.0)


def relu(z: torch.Tensor) -> torch.Tensor:
    """sites.py:221-222 build_gate('relu') -> torch.nn.ReLU."""
    return torch.relu(z)


def gelu(z: torch.Tensor) -> torch.Tensor:
    """GPT-NeoX ``act`` for the ungated A0 topology: ACT2FN['gelu'] (exact erf GELU)."""
    return torch.nn.functional.gelu(z)


def gelu_masked(z: torch.Tensor, kappa: float) -> torch.Tensor:
    """GELU(z) * [z > kappa] — the gelu-then-mask gate (strict comparison)."""
    return torch.nn.functional.gelu(z).masked_fill(~(z > kappa), 0.0)


def corner_mask(z: torch.Tensor, kappa: float, tile_tokens: int = 8, tile_features: int = 16,
                seq_len: int | None = None) -> torch.Tensor:
    """runs/063-2026-10-07-pythia14m-tile-specialized-kernel/tile_gate.py:20-29 retained_mask.

    z is [T, F] (flattened tokens) or [B, T, F].  A tile_tokens x tile_features
    tile is kept iff its top-left value is strictly greater than kappa; the
    final partial token block of each sequence is kept by its own first row.
    """
    if z.ndim == 2:
        t = z.shape[0]
        seq = t if seq_len is None else seq_len
        if t % seq:
            raise ValueError("T must be a multiple of seq_len")
        return corner_mask(z.reshape(t // seq, seq, z.shape[1]), kappa, tile_tokens, tile_features).reshape(z.shape)
    b, t, f = z.shape
    if f % tile_features:
        raise ValueError("Feature width must be divisible by tile_features")
    live = z[:, ::tile_tokens, ::tile_features] > kappa
    rows = torch.arange(t) // tile_tokens
    return live.index_select(1, rows).unsqueeze(-1).expand(b, t, f // tile_features, tile_features).reshape(b, t, f)


def corner(z: torch.Tensor, kappa: float, tile_tokens: int = 8, tile_features: int = 16,
           seq_len: int | None = None) -> torch.Tensor:
    """tile_gate.py:31-32 CornerTileThreshold.forward: zero every rejected tile."""
    return z.masked_fill(~corner_mask(z, kappa, tile_tokens, tile_features, seq_len), 0.0)


# Numbering of include/spmlp.h's SPMLP_GATE_* constants.
IDENTITY, GELU, ONE_SIDED, SYMMETRIC, RELU, GELU_MASKED, CORNER = range(7)


def apply(z: torch.Tensor, op: int, kappa: float = 0.0, seq_len: int | None = None) -> torch.Tensor:
    """Apply gate ``op`` to z (any float dtype; computed the way torch does for that dtype)."""
    if op == IDENTITY:
        return z.clone()
    if op == GELU:
        return gelu(z)
    if op == ONE_SIDED:
        return one_sided(z, kappa)
    if op == SYMMETRIC:
        return symmetric(z, kappa).clone()
    if op == RELU:
        return relu(z)
    if op == GELU_MASKED:
        return gelu_masked(z, kappa)
    if op == CORNER:
        return corner(z, kappa, 8, 16, seq_len)
    raise ValueError(f"unknown gate op {op}")


def kthvalue_threshold(z: torch.Tensor, density: float) -> float:
    """Threshold leaving about ``density`` of z above it.

    The kthvalue convention of src/sparsity_research/capture.py:142-151
    (torch.quantile rejects tensors above 2**24 elements):
    k = max(1, min(n, round(q * n))) with q = 1 - density, tau = kthvalue(k).
    """
    flat = z.reshape(-1).float()
    n = flat.numel()
    k = max(1, min(n, round((1.0 - density) * n)))
    return float(torch.kthvalue(flat, k).values)


def ulp(x: float, dtype: torch.dtype) -> float:
    """Spacing of the dtype's representable numbers just above |x| (x finite)."""
    t = torch.tensor(abs(x), dtype=dtype)
    nxt = (t.view(torch.int16) + 1).view(dtype)
    return float(nxt) - float(t)


def as_numpy_bits(t: torch.Tensor) -> np.ndarray:
    """Raw 16-bit patterns of an fp16/bf16 tensor (for bit-exact comparisons)."""
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)
