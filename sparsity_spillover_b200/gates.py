"""Gate specifications accepted at the Python boundary.

The reference describes a gate either as a spec mapping
``{"operator": ..., "kappa": ...[, "tile_tokens", "tile_features"]}``
(src/sparsity_research/sites.py:128-215, validated strictly; corner tiles:
runs/063-2026-10-07-pythia14m-tile-specialized-kernel/tile_gate.py:48-59) or as the module
installed at ``mlp.act`` (sites.py:86-107 FixedOneSidedThreshold /
FixedSymmetricThreshold, torch.nn.ReLU, tile_gate.py CornerTileThreshold; A0 keeps
GELU).  This module turns either form into the kernel's (gate_op, kappa) pair,
with kappa rounded to the activation dtype the way TensorIterator converts the
wrapped scalar (runs/063-2026-10-07-pythia14m-tile-specialized-kernel/kernel.py:17-19).
"""
from __future__ import annotations

import math
from collections.abc import Mapping
from dataclasses import dataclass
from typing import Any

import torch

from . import _lib

OPERATORS = {
    "identity": _lib.GATE_IDENTITY,
    "gelu": _lib.GATE_GELU,
    "one_sided_threshold": _lib.GATE_ONE_SIDED,
    "symmetric_threshold": _lib.GATE_SYMMETRIC,
    "relu": _lib.GATE_RELU,
    "gelu_threshold": _lib.GATE_GELU_MASKED,
    "tile_corner_threshold": _lib.GATE_CORNER,
}
_KAPPA_OPS = {"one_sided_threshold", "symmetric_threshold", "gelu_threshold", "tile_corner_threshold"}


@dataclass(frozen=True)
class GateSpec:
    """A validated gate: operator name, kernel enum, unrounded kappa."""

    operator: str
    op: int
    kappa: float = 0.0
    tile_tokens: int = 8
    tile_features: int = 16

    def kappa_for(self, dtype: torch.dtype) -> float:
        """kappa rounded to ``dtype`` (float(torch.tensor(kappa, dtype=dtype)))."""
        return float(torch.tensor(self.kappa, dtype=dtype))

    def metadata(self) -> dict[str, Any]:
        out: dict[str, Any] = {"operator": self.operator}
        if self.operator in _KAPPA_OPS:
            out["kappa"] = self.kappa
        if self.operator == "tile_corner_threshold":
            out.update(tile_tokens=self.tile_tokens, tile_features=self.tile_features)
        return out


def _nonnegative_finite(value: Any, label: str) -> float:
    # Same acceptance rule as sites.py:240-245 (_nonnegative_finite).
    if isinstance(value, bool) or not isinstance(value, int | float):
        raise ValueError(f"{label} must be a finite nonnegative number.")
    result = float(value)
    if not math.isfinite(result) or result < 0.0:
        raise ValueError(f"{label} must be a finite nonnegative number.")
    return result


def from_mapping(spec: Mapping[str, Any]) -> GateSpec:
    """Validate a gate-spec mapping (sites.py:195-214 rules, plus corner tiles)."""
    operator = spec.get("operator")
    if operator not in OPERATORS:
        raise ValueError(f"Unsupported gate operator: {operator!r}.")
    allowed = {"operator"}
    if operator in _KAPPA_OPS:
        allowed.add("kappa")
    if operator == "tile_corner_threshold":
        allowed |= {"tile_tokens", "tile_features"}
    extra = set(spec) - allowed
    if extra:
        if operator == "relu" and "kappa" in spec:
            raise ValueError("ReLU does not accept kappa.")
        raise ValueError("Unsupported gate fields: " + ", ".join(sorted(extra)))
    if operator not in _KAPPA_OPS:
        return GateSpec(operator, OPERATORS[operator])
    if "kappa" not in spec:
        raise ValueError(f"{operator} requires kappa.")
    kappa = _nonnegative_finite(spec["kappa"], "kappa")
    if operator == "tile_corner_threshold":
        tt, tf = spec.get("tile_tokens", 8), spec.get("tile_features", 16)
        for v in (tt, tf):
            if isinstance(v, bool) or not isinstance(v, int) or v <= 0:
                raise ValueError("Tile dimensions must be positive integers")
        if (tt, tf) != (8, 16):
            raise ValueError("The up-projection corner gate supports 8x16 tiles (the reference's h/z tile)")
        return GateSpec(operator, OPERATORS[operator], kappa, tt, tf)
    return GateSpec(operator, OPERATORS[operator], kappa)


def from_module(module: Any) -> GateSpec:
    """Recognise the reference's gate modules (and GELU for the ungated A0).

    The classes are matched by name and attributes so the reference package need
    not be importable where the kernels run.
    """
    name = type(module).__name__
    if isinstance(module, torch.nn.ReLU):
        return GateSpec("relu", _lib.GATE_RELU)
    if name == "FixedOneSidedThreshold":
        return GateSpec("one_sided_threshold", _lib.GATE_ONE_SIDED, _nonnegative_finite(module.kappa, "kappa"))
    if name == "FixedSymmetricThreshold":
        return GateSpec("symmetric_threshold", _lib.GATE_SYMMETRIC, _nonnegative_finite(module.kappa, "kappa"))
    if name == "CornerTileThreshold":
        return from_mapping({"operator": "tile_corner_threshold", "kappa": module.kappa,
                             "tile_tokens": module.tile_tokens, "tile_features": module.tile_features})
    if name == "GELUActivation":  # transformers ACT2FN["gelu"]: erf GELU (C or Python form)
        return GateSpec("gelu", _lib.GATE_GELU)
    if isinstance(module, torch.nn.GELU):
        if module.approximate != "none":
            raise ValueError("Only the exact (erf) GELU is supported")
        return GateSpec("gelu", _lib.GATE_GELU)
    if isinstance(module, torch.nn.Identity):
        return GateSpec("identity", _lib.GATE_IDENTITY)
    raise ValueError(f"Unsupported gate module {name}")


def resolve(gate: Any) -> GateSpec:
    """GateSpec | mapping | module | None (None = the ungated A0 GELU)."""
    if gate is None:
        return GateSpec("gelu", _lib.GATE_GELU)
    if isinstance(gate, GateSpec):
        return gate
    if isinstance(gate, Mapping):
        return from_mapping(gate)
    return from_module(gate)


HEAD_GATE_KEYS = frozenset({"operator", "kappa", "tile_tokens", "tile_features"})


def validate_head_gate(spec: Any) -> float:
    """The head-input gate of the vocabulary head: an explicit 16x16 corner gate.

    Same acceptance rule and error as the reference's head
    (runs/068-2026-10-08-pythia14m-aligned-vocabulary-tiles/inference/head.py:20-28): a mapping
    with exactly the keys operator / kappa / tile_tokens / tile_features, operator
    ``tile_corner_threshold``, 16 x 16 tiles and a finite, nonnegative, non-bool number kappa.
    Returns kappa rounded to fp32 (the certificate compares the fp32 input with it)."""
    if (not isinstance(spec, Mapping) or set(spec) != HEAD_GATE_KEYS
            or spec["operator"] != "tile_corner_threshold"
            or (spec["tile_tokens"], spec["tile_features"]) != (16, 16)
            or isinstance(spec["kappa"], bool) or not isinstance(spec["kappa"], int | float)
            or not math.isfinite(spec["kappa"]) or spec["kappa"] < 0):
        raise ValueError("An explicit unchanged corner16x16 gate is required")
    return float(torch.tensor(spec["kappa"], dtype=torch.float32))
