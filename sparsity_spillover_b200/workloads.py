"""Seeded synthetic workloads with the shapes and distributions of the benchmark configs.

The reference's trained checkpoints and its MiniPile token cache are not
available, so every config draws its inputs here (one ``torch.Generator`` seed
per config):

* cfg0  Pythia-14M MLP block, T=4096, d=128, F=512 (the CPU reference case)
* cfg1  Pythia-70M, 6 stacked MLP layers, d=512, F=2048, T=32768, fp16, density sweep
* cfg2  tile-structured h: 64x64 tiles live with probability p, GELU(N(0,1)) inside, bf16
* cfg3  Pythia-410M, 24 layers, d=1024, F=4096, T=32768 per GPU, fp16, 10% density
* cfg4  embed_out: hidden [32768, 128|512] fp16, W [50304, d], Zipf(1.1) vocabulary tiles

Weights follow GPT-NeoX's init: W_in ~ N(0, 0.02), W_out ~ N(0, 0.02/sqrt(2 L)),
biases zero; x ~ N(0, 1).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch

VOCAB = 50304


@dataclass
class MLPConfig:
    name: str
    d: int
    F: int
    layers: int
    tokens: int
    dtype: torch.dtype
    density: float
    seed: int

    @property
    def w_out_std(self) -> float:
        return 0.02 / math.sqrt(2 * self.layers)


CONFIGS = {
    "cfg0": MLPConfig("pythia14m-mlp-cpu", 128, 512, 1, 4096, torch.float32, 0.10, 1400),
    "cfg1": MLPConfig("pythia70m-mlp-6L", 512, 2048, 6, 32768, torch.float16, 0.10, 7000),
    "cfg3": MLPConfig("pythia410m-mlp-24L", 1024, 4096, 24, 32768, torch.float16, 0.10, 41000),
}


@dataclass
class MLPLayer:
    w_in: torch.Tensor
    b_in: torch.Tensor
    w_out: torch.Tensor
    b_out: torch.Tensor
    kappa: float = 0.0


@dataclass
class MLPStack:
    cfg: MLPConfig
    x: torch.Tensor
    layers: list[MLPLayer] = field(default_factory=list)


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def make_weights(cfg: MLPConfig, device, dtype: torch.dtype | None = None, seed_offset: int = 0,
                 f_slice: tuple[int, int] | None = None) -> list[MLPLayer]:
    """Per-layer weights, drawn in full and optionally sliced along d_ff (for a d_ff split)."""
    dtype = dtype or cfg.dtype
    layers = []
    for layer in range(cfg.layers):
        g = _gen(cfg.seed + 1 + layer + seed_offset, device)
        w_in = torch.randn(cfg.F, cfg.d, generator=g, device=device, dtype=torch.float32) * 0.02
        w_out = torch.randn(cfg.d, cfg.F, generator=g, device=device, dtype=torch.float32) * cfg.w_out_std
        b_in = torch.zeros(cfg.F, device=device, dtype=torch.float32)
        b_out = torch.zeros(cfg.d, device=device, dtype=torch.float32)
        if f_slice is not None:
            lo, hi = f_slice
            w_in, b_in, w_out = w_in[lo:hi].contiguous(), b_in[lo:hi].contiguous(), w_out[:, lo:hi].contiguous()
        layers.append(MLPLayer(w_in.to(dtype), b_in.to(dtype), w_out.to(dtype), b_out.to(dtype)))
    return layers


def make_input(cfg: MLPConfig, device, tokens: int | None = None, dtype: torch.dtype | None = None,
               token_offset: int = 0) -> torch.Tensor:
    """x ~ N(0,1) [tokens, d]; token_offset selects a disjoint, reproducible shard."""
    g = _gen(cfg.seed + 10_000 + token_offset, device)
    t = tokens or cfg.tokens
    return torch.randn(t, cfg.d, generator=g, device=device, dtype=torch.float32).to(dtype or cfg.dtype)


def quantile_threshold(z: torch.Tensor, density: float) -> float:
    """Threshold keeping about ``density`` of z, clamped at 0 (the reference gates
    accept only nonnegative kappa, src/sparsity_research/sites.py:240-245).

    kthvalue convention of src/sparsity_research/capture.py:142-151 (torch.quantile
    rejects more than 2**24 elements); subsampled deterministically for very
    large tensors.
    """
    flat = z.reshape(-1)
    if flat.numel() > (1 << 24):
        step = -(-flat.numel() // (1 << 24))
        flat = flat[::step]
    flat = flat.float()
    n = flat.numel()
    k = max(1, min(n, round((1.0 - density) * n)))
    return max(0.0, float(torch.kthvalue(flat.cpu(), k).values)) if not flat.is_cuda else \
        max(0.0, float(torch.sort(flat).values[k - 1]))


def tile_structured_h(tokens: int, features: int, p: float, seed: int, device, dtype=torch.bfloat16,
                      tile: int = 64) -> tuple[torch.Tensor, float]:
    """cfg2 activation: tile x tile blocks live with probability p, GELU(N(0,1)) inside.

    Returns (h, live tile fraction)."""
    g = _gen(seed, device)
    live = torch.rand(-(-tokens // tile), features // tile, generator=g, device=device) < p
    vals = torch.nn.functional.gelu(torch.randn(tokens, features, generator=g, device=device))
    mask = live.repeat_interleave(tile, 0)[:tokens].repeat_interleave(tile, 1)
    h = (vals * mask).to(dtype)
    return h, float(live.float().mean())


def corner_tile_h(tokens: int, features: int, p: float, seed: int, device, dtype=torch.float16,
                  tile_tokens: int = 8, tile_features: int = 16) -> tuple[torch.Tensor, float]:
    """h with the structure of the reference's corner-tile gate (8-token x 16-feature tiles
    kept or zeroed whole, runs/063-2026-10-07-pythia14m-tile-specialized-kernel/tile_gate.py:9-33):
    each tile kept with probability p, GELU(N(0,1)) values inside.

    Returns (h, kept tile fraction)."""
    g = _gen(seed, device)
    keep = torch.rand(-(-tokens // tile_tokens), features // tile_features, generator=g, device=device) < p
    vals = torch.nn.functional.gelu(torch.randn(tokens, features, generator=g, device=device))
    mask = keep.repeat_interleave(tile_tokens, 0)[:tokens].repeat_interleave(tile_features, 1)
    return torch.where(mask, vals, torch.zeros((), device=device)).to(dtype), float(keep.float().mean())


def zipf_active_tiles(n_tiles: int, fraction: float, seed: int, exponent: float = 1.1) -> np.ndarray:
    """Active 128-column vocabulary tiles for the tile-gated head.

    Each tile gets a seeded Zipf(exponent) score over a random rank permutation
    (with a multiplicative jitter); the round(fraction * n_tiles) best tiles are
    active.  Sorted ascending, int32."""
    rng = np.random.default_rng(seed)
    rank = rng.permutation(n_tiles) + 1
    score = rank.astype(np.float64) ** (-exponent) * rng.uniform(0.5, 1.5, n_tiles)
    count = max(1, int(round(fraction * n_tiles)))
    return np.sort(np.argsort(-score, kind="stable")[:count]).astype(np.int32)


def head_inputs(tokens: int, d: int, seed: int, device, dtype=torch.float16):
    g = _gen(seed, device)
    x = torch.randn(tokens, d, generator=g, device=device, dtype=torch.float32).to(dtype)
    w = (torch.randn(VOCAB, d, generator=g, device=device, dtype=torch.float32) * 0.02).to(dtype)
    return x, w
