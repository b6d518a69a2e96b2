"""GPT-NeoX gated MLP restated on the CPU (test oracle; see oracle/__init__.py).

GPTNeoXMLP.forward (transformers/models/gpt_neox/modeling_gpt_neox.py):
    z = dense_h_to_4h(m); h = act(z); y = dense_4h_to_h(h)
with ``act`` replaced by a gate (src/sparsity_research/pythia.py:76-77).
"""
from __future__ import annotations

import torch

from . import gates


def linear(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None, acc: torch.dtype = torch.float32) -> torch.Tensor:
    """x w^T + b in ``acc`` precision: nn.Linear's arithmetic (torch.nn.functional.linear,
    the call inside GPTNeoXMLP's dense layers) on upcast operands, without the final cast."""
    return torch.nn.functional.linear(x.to(acc), w.to(acc), None if b is None else b.to(acc))


def mlp_forward_fp32(x, w_in, b_in, w_out, b_out, gate_op: int, kappa: float, seq_len: int | None = None,
                     acc: torch.dtype = torch.float32):
    """The reference MLP in fp32 (or fp64): returns (z, h, y), all in ``acc``."""
    z = linear(x, w_in, b_in, acc)
    h = gates.apply(z, gate_op, kappa, seq_len)
    y = linear(h, w_out, b_out, acc)
    return z, h, y


def mlp_forward_dtype(x, w_in, b_in, w_out, b_out, gate_op: int, kappa: float, dtype: torch.dtype,
                      seq_len: int | None = None):
    """The MLP as an fp16/bf16 torch model computes it on CUDA: fp32 accumulation,
    one rounding per Linear, the gate on the rounded z (kappa rounded to dtype)."""
    k = gates.round_kappa(kappa, dtype)
    z = linear(x, w_in, b_in).to(dtype)
    h = gates.apply(z.float(), gate_op, k, seq_len).to(dtype) if gate_op in (gates.GELU, gates.GELU_MASKED) \
        else gates.apply(z, gate_op, k, seq_len)
    y = linear(h, w_out, b_out).to(dtype)
    return z, h, y


def down_from_h(h: torch.Tensor, w_out, b_out, residual=None, dtype: torch.dtype | None = None,
                acc: torch.dtype = torch.float32):
    """y = h w_out^T + b_out from a given (kernel-produced) h.

    With ``dtype`` set, y is rounded once to it and the residual is added the way
    the reference's joint restatement orders it (runs/027-2026-09-06-pythia14m-kernel-sparsity-characterization/
    test_adapter.py:19-25): round(round(acc + b) + r).
    """
    y = linear(h, w_out, b_out, acc)
    if dtype is None:
        return y if residual is None else y + residual.to(acc)
    y = y.to(dtype)
    if residual is not None:
        y = (y.float() + residual.float()).to(dtype)
    return y


def joint(h, z, w2, b2, wo, bo, residual, th: float, tz: float, gh: bool, gz: bool):
    """The reference's joint consumer (parallel residual of GPT-NeoX) in the activation dtype.

    runs/042-2026-09-20-pythia70m-sparse-scale/controls.py:15-27 (NativeJoint) and
    runs/027-2026-09-06-pythia14m-kernel-sparsity-characterization/test_adapter.py:19-25
    (joint_reference): gate each branch input with a one-sided threshold, round each
    branch's linear to the dtype, round the branch sum, then add the residual and round.
    """
    dtype = h.dtype
    if gh:
        h = h.masked_fill(h < th, 0)
    if gz:
        z = z.masked_fill(z < tz, 0)
    a = linear(h, w2, b2).to(dtype)
    b = linear(z, wo, bo).to(dtype)
    s = (a.float() + b.float()).to(dtype)
    return (s.float() + residual.float()).to(dtype)


def layer_norm_linear(x, gamma, beta, eps: float, w, b):
    """fp32 dense_h_to_4h(post_attention_layernorm(x)) of a GPT-NeoX layer
    (transformers GPTNeoXLayer.forward; the reference's paired LayerNorm,
    runs/035-2026-09-18-pythia70m-k050-port/kernel/norm/norm.cu:23-60, produces the
    same m).  m is kept in fp32 here, as the folded kernel does not round it."""
    m = torch.nn.functional.layer_norm(x.float(), (x.shape[-1],), None if gamma is None else gamma.float(),
                                       None if beta is None else beta.float(), eps)
    return linear(m, w, b)


def max_rel_error(actual: torch.Tensor, reference: torch.Tensor) -> float:
    """max|actual - reference| / max|reference| — the tolerance metric of the north star."""
    a, r = actual.double(), reference.double()
    denom = float(r.abs().max())
    return float((a - r).abs().max()) / (denom if denom > 0 else 1.0)


def numerical_gate(reference: torch.Tensor, actual: torch.Tensor, relative_l2: float = 0.02,
                   atol: float = 0.25, rtol: float = 0.02) -> dict:
    """rel-L2 + elementwise atol/rtol check of
    runs/025-2026-09-05-pythia-agentic-sparse-kernel-search/measurement.py:11-23."""
    reference, actual = reference.float(), actual.float()
    finite = bool(torch.isfinite(reference).all() and torch.isfinite(actual).all())
    if not finite:
        return {"pass": False, "finite": False, "relative_l2": None, "max_abs": None}
    diff = actual - reference
    rel = float(torch.linalg.vector_norm(diff) / torch.linalg.vector_norm(reference).clamp_min(1e-12))
    allclose = bool(torch.all(diff.abs() <= atol + rtol * reference.abs()))
    return {"pass": rel <= relative_l2 and allclose, "finite": True, "relative_l2": rel,
            "max_abs": float(diff.abs().max()), "elementwise_gate": allclose}
