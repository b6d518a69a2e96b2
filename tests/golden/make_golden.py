"""Generate the golden fixtures that pin the CPU oracle to the reference's own code.

Run with a checkout of the reference (thiagocmattar/sparsity-spillover), given by
--reference or by the SPARSITY_SPILLOVER_REFERENCE environment variable:

    python tests/golden/make_golden.py --reference PATH

Every fixture is produced by executing the reference's modules, never the oracle:

* gates.npz      src/sparsity_research/sites.py FixedOneSidedThreshold / FixedSymmetricThreshold /
                 build_gate('relu') on fp32/fp16/bf16 tensors with kappa ties, -0.0 and NaN;
                 runs/063-…/tile_gate.py CornerTileThreshold (8x16, 16x16, partial token blocks);
                 src/sparsity_research/capture.py clip_tensor quantile rule.
* mlp_cfg0.npz   transformers GPTNeoXMLP (hidden 128, FFN 512) with mlp.act = FixedOneSidedThreshold
                 at the 10% kthvalue threshold (config 0's block), fp32, 256 tokens.
* counts.npz     runs/042-…/tile_oracle.py counts() on structured tensors.
* joint.npz      runs/042-…/controls.py NativeJoint in bf16 with exactly representable values.
* head.npz       runs/068-…/inference/head.py pack_weight; diagnostics.py counts() certificates.
* measurement.npz runs/025-…/measurement.py paired_schedule (several counts, passes, mode lists and
                 seeds) and timing_summary on fixed synthetic samples.
* head_gate.npz  runs/068-…/inference/head.py validate_gate on accepted and rejected head-input specs.
"""
from __future__ import annotations

import argparse
import os
import importlib.util
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
R042 = "runs/042-2026-09-20-pythia70m-sparse-scale"
R063 = "runs/063-2026-10-07-pythia14m-tile-specialized-kernel"
R068 = "runs/068-2026-10-08-pythia14m-aligned-vocabulary-tiles/inference"
R025 = "runs/025-2026-09-05-pythia-agentic-sparse-kernel-search"


def load(name: str, path: Path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def bits16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy()


def gates(ref: Path) -> dict:
    from sparsity_research.capture import clip_tensor
    from sparsity_research.sites import FixedOneSidedThreshold, FixedSymmetricThreshold, build_gate

    tile_gate = load("golden_tile_gate", ref / R063 / "tile_gate.py")
    g = torch.Generator().manual_seed(20261201)
    base = torch.randn(4096, generator=g)
    base[:8] = torch.tensor([0.1, 0.5, -0.5, 0.0, -0.0, 1.0, -1.0, float("nan")])
    out: dict[str, np.ndarray] = {"z_fp32": base.numpy()}
    for dname, dtype in (("fp32", torch.float32), ("fp16", torch.float16), ("bf16", torch.bfloat16)):
        z = base.to(dtype)
        enc = (lambda t: t.numpy()) if dtype == torch.float32 else bits16
        for kappa in (0.0, 0.1, 0.5):
            tag = f"{dname}_k{kappa}"
            out[f"one_sided_{tag}"] = enc(FixedOneSidedThreshold(kappa)(z))
            out[f"symmetric_{tag}"] = enc(FixedSymmetricThreshold(kappa)(z))
        out[f"relu_{dname}"] = enc(build_gate({"operator": "relu"})(z))
    # Corner tiles on [B, T, F] with a partial final token block (T = 21) and ties at kappa.
    zc = torch.randn(2, 21, 64, generator=g)
    zc[:, ::8, ::16] = torch.tensor(0.25)
    zc[0, 8, 16] = 0.2500001
    out["corner_z"] = zc.numpy()
    for tt, tf in ((8, 16), (16, 16)):
        gate = tile_gate.CornerTileThreshold(0.25, tt, tf)
        out[f"corner_{tt}x{tf}"] = gate(zc).numpy()
        out[f"corner_mask_{tt}x{tf}"] = gate.retained_mask(zc).numpy()
    out["corner_8x16_bf16"] = bits16(tile_gate.CornerTileThreshold(0.25, 8, 16)(zc.to(torch.bfloat16)))
    # capture.py quantile clipping convention (kthvalue with k = round(q n)).
    zq = torch.randn(5000, generator=g)
    out["quantile_z"] = zq.numpy()
    out["quantile_q"] = np.array([0.9], dtype=np.float64)
    out["quantile_clipped"] = clip_tensor(zq, {"mode": "quantile", "quantile": 0.9}, torch=torch).numpy()
    return out


def mlp_cfg0() -> dict:
    import transformers
    from sparsity_research.sites import FixedOneSidedThreshold
    from transformers.models.gpt_neox.modeling_gpt_neox import GPTNeoXMLP

    cfg = transformers.GPTNeoXConfig(hidden_size=128, intermediate_size=512, hidden_act="gelu")
    torch.manual_seed(1400)
    mlp = GPTNeoXMLP(cfg).eval()
    with torch.no_grad():
        mlp.dense_h_to_4h.weight.normal_(0, 0.02)
        mlp.dense_h_to_4h.bias.normal_(0, 0.02)
        mlp.dense_4h_to_h.weight.normal_(0, 0.02 / 12 ** 0.5)
        mlp.dense_4h_to_h.bias.normal_(0, 0.02)
    x = torch.randn(256, 128)
    with torch.inference_mode():
        y_gelu = mlp(x)
        z = mlp.dense_h_to_4h(x)
        flat = z.reshape(-1)
        kappa = float(flat.kthvalue(round(0.9 * flat.numel())).values)
        mlp.act = FixedOneSidedThreshold(kappa)
        captured = {}
        mlp.act.register_forward_hook(lambda m, a, o: captured.setdefault("h", o.clone()))
        y = mlp(x)
    return {"x": x.numpy(), "w_in": mlp.dense_h_to_4h.weight.detach().numpy(),
            "b_in": mlp.dense_h_to_4h.bias.detach().numpy(), "w_out": mlp.dense_4h_to_h.weight.detach().numpy(),
            "b_out": mlp.dense_4h_to_h.bias.detach().numpy(), "kappa": np.array([kappa]), "z": z.numpy(),
            "h": captured["h"].numpy(), "y": y.numpy(), "y_gelu": y_gelu.numpy()}


def counts(ref: Path) -> dict:
    tile_oracle = load("golden_tile_oracle", ref / R042 / "tile_oracle.py")
    g = torch.Generator().manual_seed(42)
    v = torch.zeros(64, 64)
    v[8:16, :3] = 1
    v[24:32, 17:20] = 2
    v[40:48, 33] = 1  # one nonzero per row: short rows
    v[56, :] = 3
    r = (torch.rand(64, 128, generator=g) < 0.05).float() * torch.randn(64, 128, generator=g)
    out = {}
    for name, t in (("structured", v), ("sparse5", r)):
        out[f"{name}_value"] = t.numpy()
        for rows in (8, 16):
            for max_short in (2, 8):
                out[f"{name}_r{rows}_s{max_short}"] = np.array(tile_oracle.counts(t, rows, max_short=max_short))
        out[f"{name}_noskip"] = np.array(tile_oracle.counts(t, 8, skip=False))
    return out


def joint(ref: Path) -> dict:
    controls = load("golden_controls", ref / R042 / "controls.py")
    g = torch.Generator().manual_seed(7)
    m, k, n = 16, 64, 32
    # Multiples of 1/8 in [-2, 2] and weights in multiples of 1/16: every partial sum is exact in fp32.
    h = (torch.randint(-16, 17, (m, k), generator=g) / 8).bfloat16()
    z = (torch.randint(-16, 17, (m, n), generator=g) / 8).bfloat16()
    w2 = torch.nn.Linear(k, n, dtype=torch.bfloat16)
    wo = torch.nn.Linear(n, n, dtype=torch.bfloat16)
    with torch.no_grad():
        for lin in (w2, wo):
            lin.weight.copy_((torch.randint(-8, 9, lin.weight.shape, generator=g) / 16).bfloat16())
            lin.bias.copy_((torch.randint(-8, 9, lin.bias.shape, generator=g) / 16).bfloat16())
    r = (torch.randn(m, n, generator=g) * 100).bfloat16()
    out = {"h": bits16(h), "z": bits16(z), "w2": bits16(w2.weight.detach()), "b2": bits16(w2.bias.detach()),
           "wo": bits16(wo.weight.detach()), "bo": bits16(wo.bias.detach()), "r": bits16(r)}
    for gated in (False, True):
        op = controls.NativeJoint(SimpleNamespace(w2=w2, wo=wo, gh=gated, gz=gated, th=0.5, tz=0.5))
        with torch.no_grad():
            out[f"out_gated{int(gated)}"] = bits16(op(h, z, r))
    return out


def head(ref: Path) -> dict:
    sys.path.insert(0, str(ref / R068))
    try:
        head_mod = load("golden_head", ref / R068 / "head.py")
        diag = load("golden_diag", ref / R068 / "diagnostics.py")
    finally:
        sys.path.pop(0)
    tile_gate = load("golden_tile_gate_h", ref / R063 / "tile_gate.py")
    g = torch.Generator().manual_seed(68)
    out = {}
    for v in (8, 263):
        w = torch.randn(v, 128, generator=g).half()
        out[f"w_{v}"] = bits16(w)
        out[f"packed_{v}"] = bits16(head_mod.pack_weight(w))
    x = torch.randn(1, 64, 128, generator=g)
    x[:, ::16, ::16] = 0.1
    x[0, 16, 32] = float(torch.nextafter(torch.tensor(0.1), torch.tensor(1.0)))
    x[0, 32, 0] = 0.75
    gated = tile_gate.CornerTileThreshold(0.1, 16, 16)(x)
    out["x"] = x.numpy()
    out["gated"] = gated.numpy()
    c = diag.counts(gated, 0.1, 16, 256, vocabulary=263)
    for key in ("gate_tiles", "empty_gate_tiles", "issued_mma", "skipped_mma", "potential_mma"):
        out[f"count_{key}"] = np.array([c[key]])
    out["kappa_fp32"] = np.array([head_mod.validate_gate({"operator": "tile_corner_threshold", "kappa": 0.1,
                                                          "tile_tokens": 16, "tile_features": 16})])
    return out


def head_gate_cases() -> list:
    """Head-input gate specs: accepted ones and every way the reference rejects one."""
    ok = {"operator": "tile_corner_threshold", "kappa": 0.1, "tile_tokens": 16, "tile_features": 16}
    return [ok, dict(ok, kappa=0), dict(ok, kappa=3), dict(ok, kappa=1e-30), dict(ok, kappa=0.3333333333),
            dict(ok, kappa=-0.1), dict(ok, kappa=float("inf")), dict(ok, kappa=float("nan")), dict(ok, kappa=True),
            dict(ok, kappa="0.1"), dict(ok, operator="one_sided_threshold"), dict(ok, tile_tokens=8),
            dict(ok, tile_features=32), {k: v for k, v in ok.items() if k != "tile_features"},
            dict(ok, extra=1), None, [("kappa", 0.1)]]


def head_gate(ref: Path) -> dict:
    sys.path.insert(0, str(ref / R068))
    try:
        head_mod = load("golden_head_gate", ref / R068 / "head.py")
    finally:
        sys.path.pop(0)
    values = []
    for spec in head_gate_cases():
        try:
            values.append(head_mod.validate_gate(spec))
        except ValueError:
            values.append(float("nan"))  # rejected
    return {"kappa_or_nan": np.array(values, dtype=np.float64)}


# (count, passes, modes, seed) cases of the paired schedule
SCHEDULE_CASES = [(1, 1, ("native",), 0), (3, 2, ("native", "fused", "sparse"), 7),
                  (4, 3, ("dense_pytorch", "ours_rho100", "ours_rho10"), 2026), (5, 2, ("a", "b"), 123456789)]


def measurement(ref: Path) -> dict:
    meas = load("golden_measurement", ref / R025 / "measurement.py")
    out = {}
    for i, (count, passes, modes, seed) in enumerate(SCHEDULE_CASES):
        rows = meas.paired_schedule(count, passes, list(modes), seed)
        out[f"schedule{i}"] = np.array([[rep, idx] + [modes.index(m) for m in order] for rep, idx, order in rows])
    # timing_summary on fixed samples: 3 modes x 2 passes x 3 inputs, host_ms from a fixed rule
    modes = ("native", "a", "b")
    samples = []
    for rep in range(2):
        for idx in range(3):
            for j, mode in enumerate(modes):
                samples.append({"repeat": rep, "input_index": idx, "mode": mode,
                                "host_ms": 1.0 + 0.25 * j + 0.125 * idx + 0.0625 * rep * (j + 1), "cuda_ms": None})
    summary = meas.timing_summary(samples, reference="native")
    out["summary_host_ms"] = np.array([s["host_ms"] for s in samples])
    out["summary_median"] = np.array([summary[m]["median_host_ms"] for m in modes])
    out["summary_geomean"] = np.array([summary[m]["paired_geomean_speedup"] for m in modes])
    return out


def main():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", default=os.environ.get("SPARSITY_SPILLOVER_REFERENCE"),
                    help="path of a reference checkout (default: $SPARSITY_SPILLOVER_REFERENCE)")
    ap.add_argument("--only", nargs="*", help="fixture names to regenerate (default: all)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference PATH or set SPARSITY_SPILLOVER_REFERENCE")
    ref = Path(args.reference)
    sys.path.insert(0, str(ref / "src"))
    torch.set_num_threads(1)
    for name, fn in (("gates", lambda: gates(ref)), ("mlp_cfg0", mlp_cfg0), ("counts", lambda: counts(ref)),
                     ("joint", lambda: joint(ref)), ("head", lambda: head(ref)),
                     ("measurement", lambda: measurement(ref)), ("head_gate", lambda: head_gate(ref))):
        if args.only and name not in args.only:
            continue
        arrays = fn()
        np.savez_compressed(HERE / f"{name}.npz", **arrays)
        print(name, sum(a.nbytes for a in arrays.values()), "bytes")


if __name__ == "__main__":
    main()
