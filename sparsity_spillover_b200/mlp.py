"""Drop-in modules for the reference's GPT-NeoX MLP and vocabulary head.

``SparseGPTNeoXMLP`` replaces ``transformers`` GPTNeoXMLP (dense_h_to_4h -> act ->
dense_4h_to_h) whose ``act`` is one of the reference's gates
(src/sparsity_research/pythia.py:76-77).  It keeps the two nn.Linear children
under their original names, so ``state_dict`` keys are unchanged, and borrows
their weights (no copy).  Work buffers (h, tile bits) are owned by the module
and reused across calls, like the reference adapters' preallocated outputs
(runs/042-2026-09-20-pythia70m-sparse-scale/kernel/joint/candidate.py:29-30).

``SparseHead`` replaces ``embed_out`` (runs/068-2026-10-08-pythia14m-aligned-vocabulary-tiles/
inference/head.py:53-90).

Both are inference-only and CUDA-only: they raise under autograd or on CPU
tensors, as the reference adapters do (candidate.py:27).
"""
from __future__ import annotations

from typing import Any

import torch

from . import ops
from .gates import GateSpec, resolve


def _inference_guard(x: torch.Tensor) -> None:
    if torch.is_grad_enabled() and x.requires_grad:
        raise ValueError("spmlp modules are inference-only (run under torch.inference_mode or no_grad)")
    if not x.is_cuda:
        raise ValueError("spmlp modules run on CUDA tensors only")


class SparseGPTNeoXMLP(torch.nn.Module):
    """GPTNeoXMLP with a fused gate, tile bitmap and tile-skipping down-projection."""

    def __init__(self, dense_h_to_4h: torch.nn.Linear, dense_4h_to_h: torch.nn.Linear, gate: Any = None,
                 *, skip: bool = True, seq_len: int | None = None):
        super().__init__()
        self.dense_h_to_4h = dense_h_to_4h
        self.dense_4h_to_h = dense_4h_to_h
        self.gate: GateSpec = resolve(gate)
        self.skip = skip
        self.seq_len = seq_len
        self._h = self._bits = None
        self.stats: torch.Tensor | None = None

    @classmethod
    def from_mlp(cls, mlp: torch.nn.Module, *, skip: bool = True) -> "SparseGPTNeoXMLP":
        """Wrap an existing GPTNeoXMLP, reading the gate from ``mlp.act``."""
        return cls(mlp.dense_h_to_4h, mlp.dense_4h_to_h, mlp.act, skip=skip)

    def _workspace(self, tokens: int, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        f = self.dense_h_to_4h.out_features
        if self._h is None or self._h.shape[0] != tokens or self._h.device != x.device or self._h.dtype != x.dtype:
            self._h = torch.empty((tokens, f), device=x.device, dtype=x.dtype)
            self._bits = torch.empty((ops.tile_bits_size(tokens, f),), device=x.device, dtype=torch.int32)
        return self._h, self._bits

    def enable_stats(self) -> torch.Tensor:
        """Start accumulating [issued, skipped] K16 MMA steps of the down-projection."""
        dev = self.dense_4h_to_h.weight.device
        self.stats = torch.zeros(2, dtype=torch.int64, device=dev)
        return self.stats

    def forward(self, hidden_states: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
        _inference_guard(hidden_states)
        shape = hidden_states.shape
        x = hidden_states.reshape(-1, shape[-1]).contiguous()
        r = None if residual is None else residual.reshape(-1, residual.shape[-1]).contiguous()
        h, bits = self._workspace(x.shape[0], x)
        seq_len = self.seq_len or (shape[-2] if len(shape) >= 2 else x.shape[0])
        y = ops.mlp_forward(x, self.dense_h_to_4h.weight, self.dense_h_to_4h.bias, self.dense_4h_to_h.weight,
                            self.dense_4h_to_h.bias, self.gate, residual=r, skip=self.skip, h=h, bits=bits,
                            stats=self.stats, seq_len=seq_len)
        return y.view(*shape[:-1], y.shape[-1])

    def last_tile_bits(self) -> torch.Tensor | None:
        """The 16x64 tile bitmap of the last forward's h (see include/spmlp.h)."""
        return self._bits

    def extra_repr(self) -> str:
        return f"gate={self.gate.metadata()}, skip={self.skip}"


class SparseHead(torch.nn.Module):
    """embed_out replacement: dense, K-gated (corner certificates) or N-gated (vocabulary tiles)."""

    def __init__(self, linear: torch.nn.Linear, *, kappa: float | None = None, active_tiles=None,
                 dtype: torch.dtype = torch.float16, masked_value: float | None = None):
        super().__init__()
        if linear.bias is not None:
            raise ValueError("GPT-NeoX embed_out has no bias")
        if kappa is not None and active_tiles is not None:
            raise ValueError("choose the K gate (kappa) or the N gate (active_tiles)")
        self.weight = linear.weight  # original parameter, original state_dict name
        self.kappa = kappa
        self.dtype = dtype
        self.masked_value = masked_value
        w = self.weight.detach()
        # Static cast outside timing, as the reference's head does (head.py:63-66).
        self._w = w if w.dtype == dtype else w.to(dtype).contiguous()
        self._active = None
        self._inactive = None
        if active_tiles is not None:
            tiles = torch.as_tensor(active_tiles, dtype=torch.int32).flatten()
            n_tiles = self.weight.shape[0] // 128
            if tiles.numel() and (int(tiles.min()) < 0 or int(tiles.max()) >= n_tiles):
                raise ValueError("active tile index out of range")
            all_tiles = torch.ones(n_tiles, dtype=torch.bool)
            all_tiles[tiles.long()] = False
            self._active = tiles.to(self.weight.device)
            self._inactive = torch.nonzero(all_tiles).flatten().to(torch.int32).to(self.weight.device)

    def forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
        _inference_guard(hidden_states)
        shape = hidden_states.shape
        x = hidden_states.reshape(-1, shape[-1]).contiguous()
        support = None
        if self.kappa is not None:
            x, support = ops.head_prepare(x.float(), self.kappa, self.dtype)
        elif x.dtype != self.dtype:
            x = x.to(self.dtype)
        logits = ops.head_sparse(x, self._w, support=support, active_tiles=self._active)
        if self._inactive is not None and self.masked_value is not None and self._inactive.numel():
            ops.head_fill(logits, self._inactive, self.masked_value)
        return logits.view(*shape[:-1], logits.shape[-1])


def install(model: torch.nn.Module, *, skip: bool = True) -> dict[str, Any]:
    """Replace every layer's ``mlp`` of a GPTNeoXForCausalLM with SparseGPTNeoXMLP.

    The gate is read from each ``layer.mlp.act`` (the reference installs it there,
    pythia.py:76-77).  Returns metadata in the spirit of the reference installers
    (runs/042-2026-09-20-pythia70m-sparse-scale/kernel/candidate.py:14-40).
    """
    layers = getattr(getattr(model, "gpt_neox", None), "layers", None)
    if layers is None:
        raise ValueError("install() needs a GPT-NeoX model (model.gpt_neox.layers)")
    gates = []
    for layer in layers:
        if isinstance(layer.mlp, SparseGPTNeoXMLP):
            gates.append(layer.mlp.gate.metadata())
            continue
        layer.mlp = SparseGPTNeoXMLP.from_mlp(layer.mlp, skip=skip)
        gates.append(layer.mlp.gate.metadata())
    return {"mlp": "spmlp up_gate + down_sparse (sm_100a tcgen05)", "skip": skip, "gates": gates}
