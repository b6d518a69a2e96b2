"""The CPU oracle reproduces the reference's own outputs (golden fixtures made by
tests/golden/make_golden.py from the reference's modules): this pins the oracle
before any kernel is compared against it."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import bitmap as obit
from oracle import gates as og
from oracle import head as ohead
from oracle import mlp as omlp

GOLDEN = Path(__file__).resolve().parent / "golden"
DTYPES = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}


def _load(name):
    return np.load(GOLDEN / f"{name}.npz")


def _as(arr, dtype):
    t = torch.from_numpy(np.asarray(arr))
    return t if dtype == torch.float32 else t.view(dtype)


def _equal_with_nan(a: torch.Tensor, b: torch.Tensor) -> bool:
    a, b = a.float(), b.float()
    nan = torch.isnan(a)
    return bool(torch.equal(nan, torch.isnan(b)) and torch.equal(a[~nan], b[~nan]))


@pytest.mark.parametrize("dname", ["fp32", "fp16", "bf16"])
@pytest.mark.parametrize("kappa", [0.0, 0.1, 0.5])
def test_threshold_gates_match_reference_modules(dname, kappa):
    g = _load("gates")
    dtype = DTYPES[dname]
    z = torch.from_numpy(g["z_fp32"]).to(dtype)
    k = og.round_kappa(kappa, dtype)
    assert _equal_with_nan(og.one_sided(z, k), _as(g[f"one_sided_{dname}_k{kappa}"], dtype))
    assert _equal_with_nan(og.symmetric(z, k), _as(g[f"symmetric_{dname}_k{kappa}"], dtype))


@pytest.mark.parametrize("dname", ["fp32", "fp16", "bf16"])
def test_relu_matches_reference_build_gate(dname):
    g = _load("gates")
    dtype = DTYPES[dname]
    z = torch.from_numpy(g["z_fp32"]).to(dtype)
    assert _equal_with_nan(og.relu(z), _as(g[f"relu_{dname}"], dtype))


def test_one_sided_equality_survives_and_nan_is_kept():
    """sites.py:86-94 (tests/test_sites.py:28-34): z == kappa is kept; NaN < kappa is false."""
    z = torch.tensor([-2.0, 0.5, 1.0, 2.0, float("nan")])
    out = og.one_sided(z, 1.0)
    assert out[:4].tolist() == [0.0, 0.0, 1.0, 2.0] and torch.isnan(out[4])
    assert og.symmetric(torch.tensor([-1.0, -0.5, 0.5, 1.0]), 1.0).tolist() == [-1.0, 0.0, 0.0, 1.0]
    ident = torch.tensor([-1.0, 0.0, 1.0])
    assert og.symmetric(ident, 0.0) is ident


@pytest.mark.parametrize("shape", [(8, 16), (16, 16)])
def test_corner_gate_matches_reference(shape):
    g = _load("gates")
    zc = torch.from_numpy(g["corner_z"])
    tt, tf = shape
    assert torch.equal(og.corner_mask(zc, 0.25, tt, tf), torch.from_numpy(g[f"corner_mask_{tt}x{tf}"]))
    assert torch.equal(og.corner(zc, 0.25, tt, tf), torch.from_numpy(g[f"corner_{tt}x{tf}"]))
    # Flattened tokens with an explicit sequence length give the same result.
    b, t, f = zc.shape
    flat = og.corner(zc.reshape(b * t, f), 0.25, tt, tf, seq_len=t).reshape(b, t, f)
    assert torch.equal(flat, torch.from_numpy(g[f"corner_{tt}x{tf}"]))


def test_corner_gate_bf16_matches_reference():
    g = _load("gates")
    zb = torch.from_numpy(g["corner_z"]).bfloat16()
    out = og.corner(zb, og.round_kappa(0.25, torch.bfloat16))
    assert torch.equal(out, _as(g["corner_8x16_bf16"], torch.bfloat16))


def test_quantile_threshold_follows_capture_convention():
    """capture.py:142-151: zero |v| <= kthvalue(round(q n)) of |v|."""
    g = _load("gates")
    z = torch.from_numpy(g["quantile_z"])
    q = float(g["quantile_q"][0])
    tau = og.kthvalue_threshold(z.abs(), 1.0 - q)
    assert torch.equal(z.masked_fill(z.abs() <= tau, 0.0), torch.from_numpy(g["quantile_clipped"]))


def test_gpt_neox_mlp_cfg0_block_matches_reference():
    """GPTNeoXMLP(128 -> 512 -> 128) with mlp.act = FixedOneSidedThreshold(kappa): bitwise on CPU fp32."""
    g = _load("mlp_cfg0")
    t = {k: torch.from_numpy(g[k]) for k in ("x", "w_in", "b_in", "w_out", "b_out")}
    kappa = float(g["kappa"][0])
    z, h, y = omlp.mlp_forward_fp32(t["x"], t["w_in"], t["b_in"], t["w_out"], t["b_out"], og.ONE_SIDED, kappa)
    assert torch.equal(z, torch.from_numpy(g["z"]))
    assert torch.equal(h, torch.from_numpy(g["h"]))
    assert torch.equal(y, torch.from_numpy(g["y"]))
    assert abs(float((h != 0).float().mean()) - 0.1) < 0.01
    _, _, y_gelu = omlp.mlp_forward_fp32(t["x"], t["w_in"], t["b_in"], t["w_out"], t["b_out"], og.GELU, 0.0)
    assert torch.equal(y_gelu, torch.from_numpy(g["y_gelu"]))


@pytest.mark.parametrize("case", ["structured", "sparse5"])
def test_tile_occupancy_counts_match_reference(case):
    g = _load("counts")
    v = torch.from_numpy(g[f"{case}_value"])
    for rows in (8, 16):
        for max_short in (2, 8):
            assert obit.reference_counts(v, rows, max_short=max_short, n_out=512) == \
                g[f"{case}_r{rows}_s{max_short}"].tolist()
    assert obit.reference_counts(v, 8, skip=False, n_out=512) == g[f"{case}_noskip"].tolist()


@pytest.mark.parametrize("gated", [0, 1])
def test_joint_restatement_matches_reference_rounding_order(gated):
    g = _load("joint")
    bf = torch.bfloat16
    t = {k: _as(g[k], bf) for k in ("h", "z", "w2", "b2", "wo", "bo", "r")}
    out = omlp.joint(t["h"], t["z"], t["w2"], t["b2"], t["wo"], t["bo"], t["r"], 0.5, 0.5, bool(gated), bool(gated))
    assert torch.equal(out, _as(g[f"out_gated{gated}"], bf))


@pytest.mark.parametrize("v", [8, 263])
def test_head_weight_packing_matches_reference(v):
    g = _load("head")
    w = _as(g[f"w_{v}"], torch.float16)
    packed = ohead.pack_weight(w)
    assert torch.equal(packed, _as(g[f"packed_{v}"], torch.float16).reshape(packed.shape))
    inverse = ohead.unpack_weight(packed)
    assert torch.equal(inverse[:v], w) and inverse[v:].count_nonzero() == 0


def test_head_certificates_match_reference_counts():
    """runs/068-…/inference/diagnostics.py counts(): fp32 corners > kappa decide the 16x16 tiles."""
    g = _load("head")
    x = torch.from_numpy(g["x"]).reshape(-1, 128)
    gated = torch.from_numpy(g["gated"]).reshape(-1, 128)
    kappa = float(g["kappa_fp32"][0])
    live = ohead.support_mask(x, kappa)
    assert int(live.size) == int(g["count_gate_tiles"][0])
    assert int((~live).sum()) == int(g["count_empty_gate_tiles"][0])
    issued_per_tile = int(g["count_issued_mma"][0]) // max(1, int(live.sum()))
    assert int(live.sum()) * issued_per_tile == int(g["count_issued_mma"][0])
    prepared, _ = ohead.prepare(x, kappa, torch.float32)
    assert torch.equal(prepared, gated)
