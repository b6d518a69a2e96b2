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

``JointConsumer`` replaces the reference's joint consumer of a parallel-residual
layer (``Joint`` of runs/026-2026-09-06-pythia14m-fused-sparse-kernel/autoresearch/
candidates/k018/candidate.py:25-46 and runs/027-2026-09-06-pythia14m-kernel-sparsity-
characterization/adapter.py:35-51): ``joint(h, z, residual)`` returns
``round(round(round(W2 h + b2) + round(Wo z + bo)) + residual)`` with the h and z
gates applied first.  ``install_joint(model)`` rewires every layer's forward the way
the reference's adapter does (k018 candidate.py:48-56, 69-75), with the up projection,
gate and bitmap fused by ``up_gate``.

Both are inference-only and CUDA-only: they raise under autograd or on CPU
tensors, as the reference adapters do (candidate.py:27).
"""
from __future__ import annotations

from typing import Any

import torch

from types import MethodType

from . import _lib, gates, ops
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
                 dtype: torch.dtype = torch.float16, masked_value: float | None = None, skip: bool = True):
        super().__init__()
        if linear.bias is not None:
            raise ValueError("GPT-NeoX embed_out has no bias")
        if kappa is not None and active_tiles is not None:
            raise ValueError("choose the K gate (kappa) or the N gate (active_tiles)")
        self.weight = linear.weight  # original parameter, original state_dict name
        self.kappa = kappa
        self.skip = skip  # K gate: skip dead K16 steps (False: certificates applied, every step issued)
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

    @classmethod
    def from_spec(cls, linear: torch.nn.Linear, spec, *, skip: bool = True,
                  dtype: torch.dtype = torch.float16) -> "SparseHead":
        """The reference head's constructor form, Head(linear, spec, skip=...)
        (runs/068-2026-10-08-pythia14m-aligned-vocabulary-tiles/inference/head.py:48-60): spec is
        the explicit 16x16 corner gate of the head input (gates.validate_head_gate)."""
        return cls(linear, kappa=gates.validate_head_gate(spec), dtype=dtype, skip=skip)

    def forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
        _inference_guard(hidden_states)
        shape = hidden_states.shape
        x = hidden_states.reshape(-1, shape[-1]).contiguous()
        support = None
        if self.kappa is not None:
            x, support = ops.head_prepare(x.float(), self.kappa, self.dtype)
            if not self.skip:
                support = None  # the zeroed tiles contribute exact zeros either way
        elif x.dtype != self.dtype:
            x = x.to(self.dtype)
        logits = ops.head_sparse(x, self._w, support=support, active_tiles=self._active)
        if self._inactive is not None and self.masked_value is not None and self._inactive.numel():
            ops.head_fill(logits, self._inactive, self.masked_value)
        return logits.view(*shape[:-1], logits.shape[-1])


HEAD_MODES = ("dense", "custom_no_skip", "custom_sparse")


def install_head(model: torch.nn.Module, mode: str, config: dict[str, Any] | None = None) -> dict[str, Any]:
    """Replace ``model.embed_out`` as the reference's head installer does
    (runs/068-2026-10-08-pythia14m-aligned-vocabulary-tiles/inference/head.py:93-112).

    mode ``dense``: every logit from the sm_100a kernel, no gate; ``custom_no_skip``: the
    head input's 16x16 corner certificates (``model.config.head_input_gate``) zero dead
    tiles, every K16 step is issued; ``custom_sparse``: the same, dead K16 steps skipped.
    ``config`` may carry the reference's consumer tile (``kernel_tile_tokens`` 16,
    ``kernel_tile_vocabulary`` 128/256/512), validated as there and recorded; the kernel's
    own tile is 128 tokens x 128 vocabulary columns (two per CTA pair for d >= 256, dense)."""
    if mode not in HEAD_MODES:
        raise ValueError(mode)
    spec = getattr(model.config, "head_input_gate", None)
    config = dict(config or {})
    tile = (config.get("kernel_tile_tokens", 16), config.get("kernel_tile_vocabulary", 256))
    if tile[0] != 16 or tile[1] not in (128, 256, 512):
        raise ValueError("Unsupported consumer tile")
    linear = model.embed_out
    if isinstance(linear, SparseHead):
        raise ValueError("embed_out is already replaced")
    if mode == "dense":
        head = SparseHead(linear)
    else:
        head = SparseHead.from_spec(linear, spec, skip=mode == "custom_sparse")
    model.embed_out = head
    return {"mode": mode, "gate": None if mode == "dense" else dict(spec), "gate_materialized": mode != "dense",
            "parameters": "unchanged", "projection": "fp16 inputs and weights, fp32 accumulation, fp16 logits",
            "static_weight_preparation": "one fp16 cast outside timing, no packed copy (w_vocab is K-major)",
            "certificate": None if mode == "dense" else "fp32 corner > fp32 threshold before the cast",
            "consumer_tile": [tile[0], tile[1], 16]}


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


def _branch_gate(module: Any, allowed: tuple[int, ...]) -> GateSpec | None:
    """The reference joint's input gate for one branch, or None when it has none."""
    if module is None:
        return None
    try:
        spec = resolve(module)
    except ValueError:
        return None
    return spec if spec.op in allowed else None


class JointConsumer:
    """The joint consumer of one parallel-residual GPT-NeoX layer, in one sm_100a kernel.

    Mirrors the reference's ``Joint(layer)``: ``w2`` is ``layer.mlp.dense_4h_to_h``,
    ``wo`` is ``layer.attention.dense``; ``gh`` / ``th`` come from ``layer.mlp.act``
    (a one-sided threshold or ReLU) and ``gz`` / ``tz`` from ``layer.attention.z_gate``
    (a one-sided threshold), as in runs/027-2026-09-06-pythia14m-kernel-sparsity-
    characterization/adapter.py:37-41.  Output and gate buffers are owned by the
    object and reused across calls.  Inference only, CUDA only, fp16 or bf16.
    """

    def __init__(self, layer: torch.nn.Module, *, skip: bool | str = True):
        self.w2 = layer.mlp.dense_4h_to_h
        self.wo = layer.attention.dense
        self.h_gate = _branch_gate(getattr(layer.mlp, "act", None), (_lib.GATE_ONE_SIDED, _lib.GATE_RELU))
        self.z_gate = _branch_gate(getattr(layer.attention, "z_gate", None), (_lib.GATE_ONE_SIDED,))
        self.gh, self.gz = self.h_gate is not None, self.z_gate is not None
        self.th = self.h_gate.kappa if self.gh else 0.0
        self.tz = self.z_gate.kappa if self.gz else 0.0
        self.skip = skip
        self.stats: torch.Tensor | None = None
        self._buffers: dict[str, torch.Tensor] = {}
        # Set by install_joint: the up projection run by the fused layer forward.
        self.up: torch.nn.Linear | None = None
        self.up_gate: GateSpec | None = None
        self.folded: ops.FoldedLayerNorm | None = None

    def _buffer(self, name: str, shape: tuple[int, ...], like: torch.Tensor, dtype: torch.dtype | None = None):
        dtype = dtype or like.dtype
        buf = self._buffers.get(name)
        if buf is None or buf.shape != shape or buf.dtype != dtype or buf.device != like.device:
            buf = self._buffers[name] = torch.empty(shape, device=like.device, dtype=dtype)
        return buf

    def enable_stats(self) -> torch.Tensor:
        """Start accumulating [issued, skipped] K16 MMA steps of the h branch."""
        self.stats = torch.zeros(2, dtype=torch.int64, device=self.w2.weight.device)
        return self.stats

    def __call__(self, h: torch.Tensor, z: torch.Tensor, residual: torch.Tensor) -> torch.Tensor:
        """Reference contract: h is the ungated up-projection output, z the ungated
        attention context; both gates are applied here."""
        _inference_guard(h)
        h2 = h.reshape(-1, h.shape[-1]).contiguous()
        t, f = h2.shape
        bits = self._buffer("bits", (ops.tile_bits_size(t, f),), h2, torch.int32)
        if self.gh:
            h2 = ops.gate(h2, self.h_gate, out=self._buffer("h", (t, f), h2), bits=bits)
        else:
            ops.tile_bits_from_h(h2, bits)
        return self.forward_gated(h2, bits, z, residual)

    def forward_gated(self, h: torch.Tensor, bits: torch.Tensor | None, z: torch.Tensor,
                      residual: torch.Tensor) -> torch.Tensor:
        """h already gated, with its tile bitmap (e.g. from ``ops.up_gate``)."""
        _inference_guard(z)
        z2 = z.reshape(-1, z.shape[-1]).contiguous()
        r = residual.reshape(-1, residual.shape[-1]).contiguous()
        if self.gz:
            z2 = ops.gate(z2, self.z_gate, out=self._buffer("z", tuple(z2.shape), z2))
        out = self._buffer("out", tuple(r.shape), r)
        ops.joint(h, bits, z2, self.w2.weight, self.w2.bias, self.wo.weight, self.wo.bias, r, skip=self.skip,
                  out=out, stats=self.stats)
        return out.view_as(residual)


def _joint_layer_forward(self, hidden_states, attention_mask=None, position_ids=None, use_cache=False,
                         layer_past=None, position_embeddings=None, **kwargs):
    """GPTNeoXLayer.forward with parallel residual, fused as in the reference's
    layer_forward (k018 candidate.py:48-56): attention up to its context z, the
    fused up projection + gate + bitmap, then the joint consumer."""
    if use_cache or layer_past is not None or self.training:
        raise ValueError("the joint consumer runs uncached inference only")
    z, _ = self.attention(self.input_layernorm(hidden_states), attention_mask=attention_mask,
                          position_ids=position_ids, layer_past=None, use_cache=False,
                          position_embeddings=position_embeddings, **kwargs)
    joint = self._spmlp_joint
    shape = hidden_states.shape
    seq_len = shape[-2] if len(shape) >= 2 else None
    if joint.folded is not None:
        # post_attention_layernorm folded into the up projection: read the residual stream itself.
        x = hidden_states.reshape(-1, shape[-1]).contiguous()
        t, f = x.shape[0], joint.up.out_features
        h = joint._buffer("h_up", (t, f), x)
        bits = joint._buffer("bits_up", (ops.tile_bits_size(t, f),), x, torch.int32)
        stats = (joint._buffer("ln_mean", (t,), x, torch.float32), joint._buffer("ln_rstd", (t,), x, torch.float32))
        ops.row_stats(x, joint.folded.eps, *stats)
        ops.up_gate_ln(x, joint.folded, joint.up_gate, h=h, bits=bits, seq_len=seq_len, stats=stats)
    else:
        m = self.post_attention_layernorm(hidden_states)
        x = m.reshape(-1, shape[-1]).contiguous()
        t, f = x.shape[0], joint.up.out_features
        h = joint._buffer("h_up", (t, f), x)
        bits = joint._buffer("bits_up", (ops.tile_bits_size(t, f),), x, torch.int32)
        ops.up_gate(x, joint.up.weight, joint.up.bias, joint.up_gate, h=h, bits=bits, seq_len=seq_len)
    return joint.forward_gated(h, bits, z, hidden_states)


def install_joint(model: torch.nn.Module, *, skip: bool | str = True, fuse_layernorm: bool = False) -> dict[str, Any]:
    """Fuse every parallel-residual layer's output side into one joint kernel.

    Per layer, as the reference's Adapter.install (k018 candidate.py:69-75): the
    attention's dense projection becomes the joint's z branch (``attention.dense``
    is replaced by Identity, so attention returns its context), the MLP's down
    projection its h branch, and ``layer.forward`` calls up_gate then the joint.
    The gate of h stays ``layer.mlp.act`` (applied by up_gate); a one-sided
    ``attention.z_gate`` is applied to z by the joint and bypassed inside attention.
    With ``fuse_layernorm`` the MLP's post_attention_layernorm is folded into the up
    projection (``ops.FoldedLayerNorm``, prepared here once), so its output is never
    materialised; z then skips the rounding of the normalized activation.
    """
    layers = getattr(getattr(model, "gpt_neox", None), "layers", None)
    if layers is None:
        raise ValueError("install_joint() needs a GPT-NeoX model (model.gpt_neox.layers)")
    gates = []
    for layer in layers:
        if not getattr(layer, "use_parallel_residual", False):
            raise ValueError("the joint consumer needs GPT-NeoX's parallel residual")
        mlp = layer.mlp
        joint = JointConsumer(layer, skip=skip)
        joint.up = mlp.dense_h_to_4h
        joint.up_gate = mlp.gate if isinstance(mlp, SparseGPTNeoXMLP) else resolve(getattr(mlp, "act", None))
        joint.folded = (ops.FoldedLayerNorm.from_modules(layer.post_attention_layernorm, joint.up)
                        if fuse_layernorm else None)
        layer._spmlp_joint = joint
        layer.attention.dense = torch.nn.Identity()
        if joint.gz:
            layer.attention.z_gate.forward = MethodType(lambda self, x: x, layer.attention.z_gate)
        layer.forward = MethodType(_joint_layer_forward, layer)
        gates.append({"h": joint.up_gate.metadata(), "z": joint.z_gate.metadata() if joint.gz else None})
    return {"joint": "spmlp up_gate + joint (sm_100a tcgen05)", "skip": skip, "fuse_layernorm": fuse_layernorm,
            "gates": gates}
