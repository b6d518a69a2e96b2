"""Benchmark of the B200 sparse gated MLP (driver contract: one JSON line on rank 0).

Workload (the headline configuration): Pythia-70M MLP, 6 stacked layers, d=512, F=2048,
T=32768 tokens per GPU, fp16, one-sided threshold gate at 10% element density
(kappa calibrated per layer by the kthvalue rule).  Layers are chained through
the parallel residual, x_{l+1} = round(x_l + MLP_l(x_l)), which the down-projection
kernel fuses.  One step = the 6-layer forward over one batch of tokens.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs under torchrun, one rank per GPU: tokens are sharded (each rank owns a
disjoint 32768-token batch, same weights), no collective on the data path; time
is the max over ranks.  ``--impl reference`` times the reference's CPU path (the
oracle restatement of GPTNeoXMLP + FixedOneSidedThreshold in fp32) on the host.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "gated-MLP fwd tokens/s at 1/2/4/8 B200 and speedup vs dense GEMM by density"
DENSITY = 0.10
WORKLOAD = ("cfg1: Pythia-70M gated MLP, 6 stacked layers, d=512 F=2048, T=32768/GPU, "
            "one-sided threshold gate at 10% element density, residual chained")
PEAKS_FILE = ROOT / "MEASURED_PEAKS.json"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# DRAM bytes per launch from one ncu capture of the same layer shape
# (dram__bytes_read.sum + dram__bytes_write.sum; profiles/gemm_up_down_cfg1.md).
NCU_TRAFFIC_BYTES: dict[str, float | None] = {"up_gate": 116.4e6, "down_sparse": 192.0e6}


def peaks() -> tuple[dict, str]:
    if PEAKS_FILE.exists():
        return json.loads(PEAKS_FILE.read_text()), "measured"
    return dict(FALLBACK_PEAKS), "fallback"


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 20 ms during the timed regions."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus: list[int]):
        self.gpus = gpus
        self.proc = None
        self.lines: list[str] = []
        self._thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "20",
                 "-i", ",".join(str(g) for g in self.gpus)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
            return
        self._thread = threading.Thread(target=self._read, daemon=True)
        self._thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, power, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        loaded = [s for s, p in zip(sm, power) if p > 200] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": max(power)}


# ---------------------------------------------------------------- distributed plumbing
def dist_setup(backend: str):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        import datetime

        kwargs = {"timeout": datetime.timedelta(seconds=120)}
        if backend == "nccl":
            torch.cuda.set_device(local)
            kwargs["device_id"] = torch.device("cuda", local)
        dist.init_process_group(backend, **kwargs)
    return world, rank, local


def max_over_ranks(value: float, world: int, device) -> float:
    if world == 1:
        return value
    import torch
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int, device=None):
    if world > 1:
        import torch.distributed as dist

        if device is not None:
            dist.barrier(device_ids=[device.index])
        else:
            dist.barrier()


# ---------------------------------------------------------------- our arm
class Stack:
    """Weights, calibrated gates and activation buffers of the 6-layer workload on one GPU."""

    def __init__(self, device, rank: int, density: float, cfg_name: str = "cfg1"):
        import torch

        from sparsity_spillover_b200 import ops, workloads

        self.cfg = cfg = workloads.CONFIGS[cfg_name]
        self.device = device
        self.layers = workloads.make_weights(cfg, device)
        self.x0 = workloads.make_input(cfg, device, token_offset=rank)
        t, d, f = cfg.tokens, cfg.d, cfg.F
        self.xs = [self.x0] + [torch.empty(t, d, dtype=cfg.dtype, device=device) for _ in range(cfg.layers)]
        self.h = torch.empty(t, f, dtype=cfg.dtype, device=device)
        self.bits = torch.empty(ops.tile_bits_size(t, f), dtype=torch.int32, device=device)
        self.stats = torch.zeros(2, dtype=torch.int64, device=device)
        self.gates = []
        z = torch.empty(t, f, dtype=cfg.dtype, device=device)
        for i, layer in enumerate(self.layers):
            ops.up_gate(self.xs[i], layer.w_in, layer.b_in, {"operator": "identity"}, h=self.h, bits=self.bits,
                        z_out=z)
            kappa = workloads.quantile_threshold(z, density) if density < 1.0 else None
            gate = {"operator": "one_sided_threshold", "kappa": kappa} if kappa is not None else {"operator": "identity"}
            self.gates.append(gate)
            self.layer(i, stats=self.stats)
        del z
        torch.cuda.synchronize(device)
        self.density = self._density()

    def _density(self) -> float:
        # Element density of the last layer's h (calibration check).
        return float((self.h != 0).float().mean())

    def layer(self, i: int, stats=None, events=None):
        from sparsity_spillover_b200 import ops

        L = self.layers[i]
        if events is not None:
            events[0].record()
        ops.up_gate(self.xs[i], L.w_in, L.b_in, self.gates[i], h=self.h, bits=self.bits)
        if events is not None:
            events[1].record()
        ops.down_sparse(self.h, self.bits, L.w_out, L.b_out, self.xs[i], y=self.xs[i + 1], stats=stats)
        if events is not None:
            events[2].record()

    def step(self, events=None):
        for i in range(len(self.layers)):
            self.layer(i, events=None if events is None else events[i])
        return self.xs[-1]


def dense_reference_step(stack: Stack, x=None):
    """The same 6-layer forward as stock PyTorch runs it on CUDA: cuBLAS Linear, masked_fill gate,
    residual add (the reference's own GPU path for the block, without custom kernels)."""
    import torch

    x = stack.x0 if x is None else x
    for layer, gate in zip(stack.layers, stack.gates):
        z = torch.nn.functional.linear(x, layer.w_in, layer.b_in)
        if gate["operator"] == "one_sided_threshold":
            z = z.masked_fill(z < gate["kappa"], 0.0)
        x = torch.nn.functional.linear(z, layer.w_out, layer.b_out) + x
    return x


def graph_of(fn, device):
    """Capture fn() once as a CUDA graph on a side stream."""
    import torch

    fn()
    torch.cuda.synchronize(device)
    g = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        with torch.cuda.graph(g, stream=side):
            fn()
    torch.cuda.current_stream(device).wait_stream(side)
    return g


def density_sweep(device, densities=(1.0, 0.5, 0.25, 0.1, 0.05), steps=5) -> list[dict]:
    """cfg1 at each density: our 6-layer step vs the stock PyTorch forward (both graph-replayed)."""
    import torch

    rows = []
    for rho in densities:
        st = Stack(device, 0, rho)
        g_ours = graph_of(st.step, device)
        g_ref = graph_of(lambda: dense_reference_step(st), device)
        t_ours = time_device(g_ours.replay, steps, device)
        t_ref = time_device(g_ref.replay, steps, device)
        issued, skipped = st.stats.cpu().tolist()
        rows.append({"density_target": rho, "density_measured": round(st.density, 4),
                     "tokens_per_s": st.cfg.tokens / t_ours, "dense_pytorch_tokens_per_s": st.cfg.tokens / t_ref,
                     "speedup_vs_dense_pytorch": t_ref / t_ours, "skipped_k16_fraction": skipped / max(1, issued + skipped)})
        del g_ours, g_ref, st
        torch.cuda.empty_cache()
    base = rows[0]["tokens_per_s"]
    for r in rows:
        r["speedup_vs_ours_at_100pct"] = r["tokens_per_s"] / base
    return rows


def paired_cfg1(device, passes: int = 3, n_inputs: int = 4, warmups: int = 2) -> dict:
    """cfg1 under the reference's paired, rotating-input latency protocol
    (runs/025-…/measurement.py:26-97): four seeded input batches, every (pass, input)
    block running {stock PyTorch at rho = 0.1, ours at rho = 1, ours at rho = 0.1} in a
    shuffled order, eager calls, synchronised host latency as the primary figure and
    the paired geometric-mean speed-up over stock PyTorch."""
    from sparsity_spillover_b200 import measurement, workloads

    stacks = {"ours_rho10": Stack(device, 0, DENSITY), "ours_rho100": Stack(device, 0, 1.0)}
    cfg = stacks["ours_rho10"].cfg
    inputs = [workloads.make_input(cfg, device, token_offset=1000 + i) for i in range(n_inputs)]
    modes = ["dense_pytorch", "ours_rho100", "ours_rho10"]
    current = {"mode": modes[0]}

    def set_mode(mode):
        current["mode"] = mode

    def forward(x):
        if current["mode"] == "dense_pytorch":
            return dense_reference_step(stacks["ours_rho10"], x)
        st = stacks[current["mode"]]
        st.xs[0] = x
        return st.step()

    samples = measurement.paired_timing(forward, set_mode, inputs, modes=modes, passes=passes, warmups=warmups,
                                        seed=2026)
    return {"protocol": f"paired rotating inputs: {n_inputs} inputs x {passes} passes, shuffled mode order, "
                        f"{warmups} warm-ups per mode, eager calls, seed 2026",
            "density_measured": {k: round(v.density, 4) for k, v in stacks.items()},
            "summary": measurement.timing_summary(samples, reference="dense_pytorch", tokens_per_call=cfg.tokens)}


def tile_structured(device, steps=10) -> list[dict]:
    """cfg2: tile-structured h (64x64 tiles live with probability p), bf16, T=65536: the
    skipping down-projection against its dense mode and cuBLAS."""
    import torch

    from sparsity_spillover_b200 import ops, workloads

    rows = []
    for d, f in ((256, 1024), (512, 2048)):
        g = torch.Generator(device=device).manual_seed(20 + d)
        w = (torch.randn(d, f, generator=g, device=device) * 0.02).bfloat16()
        for p in (0.5, 0.2, 0.1):
            h, frac = workloads.tile_structured_h(65536, f, p, seed=int(p * 100) + d, device=device)
            bits = ops.tile_bits_from_h(h)
            y = torch.empty(65536, d, dtype=torch.bfloat16, device=device)
            stats = {}
            times = {}
            for mode in ("fine", True, False):
                st = torch.zeros(2, dtype=torch.int64, device=device)
                ops.down_sparse(h, bits, w, None, skip=mode, y=y, stats=st)
                stats[str(mode)] = st.cpu().tolist()
                times[str(mode)] = time_device(lambda: ops.down_sparse(h, bits, w, None, skip=mode, y=y), steps, device)
            t_cublas = time_device(lambda: torch.nn.functional.linear(h, w), steps, device)
            t_bits = time_device(lambda: ops.tile_bits_from_h(h, bits), steps, device)
            fi = stats["fine"]
            rows.append({"d": d, "F": f, "p": p, "live_tile_fraction": round(frac, 4),
                         "down_fine_us": times["fine"] * 1e6, "down_coarse_us": times["True"] * 1e6,
                         "down_dense_us": times["False"] * 1e6, "cublas_us": t_cublas * 1e6, "bitmap_us": t_bits * 1e6,
                         "skipped_k16_fraction_fine": fi[1] / max(1, fi[0] + fi[1]),
                         "speedup_fine_vs_dense": times["False"] / times["fine"],
                         "speedup_fine_vs_cublas": t_cublas / times["fine"], "ideal_speedup": 1.0 / max(frac, 1e-9)})
            del h, bits, y
        torch.cuda.empty_cache()
    return rows


def corner_tiles_cfg1(device, steps=10) -> list[dict]:
    """The down projection on h with the reference's corner-tile structure (8-token x
    16-feature tiles kept whole with probability p; cfg1 layer shape T=32768, d=512,
    F=2048, fp16): every mode, with the skipped K16 fraction against the ideal (the
    dead 16x16 granules), and cuBLAS."""
    import torch

    from sparsity_spillover_b200 import ops, workloads

    t, d, f = 32768, 512, 2048
    g = torch.Generator(device=device).manual_seed(61)
    w = (torch.randn(d, f, generator=g, device=device) * 0.02).half()
    y = torch.empty(t, d, dtype=torch.float16, device=device)
    rows = []
    for p in (0.01, 0.02, 0.05):
        h, kept = workloads.corner_tile_h(t, f, p, seed=int(p * 1000) + 3, device=device)
        b64, b16 = ops.tile_bits_from_h(h), ops.tile_bits16_from_h(h)
        import numpy as np

        live16 = float(np.unpackbits(b16.cpu().numpy().view(np.uint8)).mean())  # F/16 = 128: every bit is a tile
        density = float((h != 0).float().mean())
        # ideal: the skipped fraction if every dead 16x16 tile (the finest granule a 16-row
        # MMA could skip) were skipped, and the element-level zero fraction
        row = {"p": p, "kept_tile_fraction": round(kept, 4), "element_density": round(density, 4),
               "ideal_skipped_fraction_16x16": 1.0 - live16, "ideal_skipped_fraction_elements": 1.0 - density}
        for mode in (False, True, "fine", "compact", "compact_fine"):
            bits = b16 if isinstance(mode, str) and mode.startswith("compact") else b64
            st = torch.zeros(2, dtype=torch.int64, device=device)
            ops.down_sparse(h, bits, w, None, skip=mode, y=y, stats=st)
            issued, skipped = st.tolist()
            name = {False: "dense", True: "coarse"}.get(mode, mode)
            row[f"{name}_us"] = time_device(lambda: ops.down_sparse(h, bits, w, None, skip=mode, y=y), steps,
                                            device) * 1e6
            row[f"{name}_skipped_k16_fraction"] = skipped / max(1, issued + skipped)
        row["cublas_us"] = time_device(lambda: torch.nn.functional.linear(h, w), steps, device) * 1e6
        best = min(("fine", "compact_fine", "coarse", "dense", "compact"), key=lambda m: row[f"{m}_us"])
        row["best_mode"] = best
        row["best_speedup_vs_cublas"] = row["cublas_us"] / row[f"{best}_us"]
        rows.append(row)
        del h, b64, b16
    return rows


def cfg3_410m(device, steps=3) -> dict:
    """cfg3: Pythia-410M shape, 24 layers, d=1024 F=4096, T=32768 per GPU, fp16, 10% density."""
    import torch

    st = Stack(device, 0, DENSITY, cfg_name="cfg3")
    g_ours = graph_of(st.step, device)
    g_ref = graph_of(lambda: dense_reference_step(st), device)
    t_ours = time_device(g_ours.replay, steps, device)
    t_ref = time_device(g_ref.replay, steps, device)
    cfg = st.cfg
    flop = cfg.layers * 2 * (2.0 * cfg.tokens * cfg.d * cfg.F)
    out = {"tokens_per_s": cfg.tokens / t_ours, "ms_per_step": t_ours * 1e3, "dense_pytorch_tokens_per_s": cfg.tokens / t_ref,
           "speedup_vs_dense_pytorch": t_ref / t_ours, "executed_tflops": flop / t_ours / 1e12,
           "density_measured": round(st.density, 4)}
    del g_ours, g_ref, st
    torch.cuda.empty_cache()
    return out


def head_bench(device, steps=5) -> list[dict]:
    """cfg4: embed_out [32768, d] x [d, 50304] fp16 with Zipf(1.1)-chosen active 128-column tiles."""
    import torch

    from sparsity_spillover_b200 import ops, workloads

    rows = []
    t_tokens = 32768
    for d in (128, 512):
        x, w = workloads.head_inputs(t_tokens, d, seed=40 + d, device=device)
        logits = torch.empty(t_tokens, workloads.VOCAB, dtype=torch.float16, device=device)
        t_dense = time_device(lambda: ops.head_sparse(x, w, logits=logits), steps, device)
        t_cublas = time_device(lambda: torch.nn.functional.linear(x, w), steps, device)
        for frac in (0.05, 0.1, 0.25):
            tiles = torch.from_numpy(workloads.zipf_active_tiles(workloads.VOCAB // 128, frac, seed=7)).to(device)
            t_n = time_device(lambda: ops.head_sparse(x, w, active_tiles=tiles, logits=logits), steps, device)
            rows.append({"d": d, "active_fraction": frac, "n_gated_us": t_n * 1e6, "dense_us": t_dense * 1e6,
                         "cublas_us": t_cublas * 1e6, "speedup_vs_cublas": t_cublas / t_n,
                         "logit_write_gbs": t_tokens * tiles.numel() * 128 * 2 / t_n / 1e9})
        if d == 128:
            # the reference's own head mode: 16x16 corner certificates of the fp32 head input
            # (runs/068-…/inference/head.cu), dead K16 steps skipped per 128-token block
            g = torch.Generator(device=device).manual_seed(68)
            xf = torch.randn(t_tokens, d, generator=g, device=device)
            for kappa in (0.0, 1.0, 2.0):
                xh, support = ops.head_prepare(xf, kappa, torch.float16)
                st = torch.zeros(2, dtype=torch.int64, device=device)
                ops.head_sparse(xh, w, support=support, logits=logits, stats=st)
                issued, skipped = st.tolist()
                t_prep = time_device(lambda: ops.head_prepare(xf, kappa, torch.float16, x_out=xh, support=support),
                                     steps, device)
                t_k = time_device(lambda: ops.head_sparse(xh, w, support=support, logits=logits), steps, device)
                rows.append({"d": d, "mode": "k_gate_corner16x16", "kappa": kappa,
                             "skipped_k16_fraction": skipped / max(1, issued + skipped),
                             "prepare_us": t_prep * 1e6, "k_gated_us": t_k * 1e6, "dense_us": t_dense * 1e6,
                             "cublas_us": t_cublas * 1e6, "speedup_vs_cublas": t_cublas / (t_prep + t_k)})
        del x, w, logits
        torch.cuda.empty_cache()
    return rows


def layernorm_fold_cfg1(device, steps: int = 10) -> dict:
    """post_attention_layernorm + up projection + gate on a cfg1 layer (T=32768, d=512,
    F=2048, fp16): torch's LayerNorm followed by up_gate, against the LayerNorm folded
    into the up projection (row statistics + up_gate_ln; the normalized activation is
    never written); each captured as a CUDA graph."""
    import torch

    from sparsity_spillover_b200 import ops, workloads

    cfg = workloads.CONFIGS["cfg1"]
    layer = workloads.make_weights(cfg, device)[0]
    x = workloads.make_input(cfg, device) + 2.0
    ln = torch.nn.LayerNorm(cfg.d, eps=1e-5).to(device=device, dtype=cfg.dtype)
    with torch.no_grad():
        ln.weight.normal_(1.0, 0.1)
        ln.bias.normal_(0.0, 0.1)
    gate = {"operator": "one_sided_threshold", "kappa": 0.05}
    fold = ops.FoldedLayerNorm(ln.weight, ln.bias, ln.eps, layer.w_in, layer.b_in)
    t, f = x.shape[0], cfg.F
    h = torch.empty(t, f, dtype=cfg.dtype, device=device)
    bits = torch.empty(ops.tile_bits_size(t, f), dtype=torch.int32, device=device)
    stats = (torch.empty(t, device=device), torch.empty(t, device=device))

    def unfused():
        ops.up_gate(ln(x), layer.w_in, layer.b_in, gate, h=h, bits=bits)

    def fused():
        ops.row_stats(x, ln.eps, *stats)
        ops.up_gate_ln(x, fold, gate, h=h, bits=bits, stats=stats)

    t_un = time_device(graph_of(unfused, device).replay, steps, device)
    t_fu = time_device(graph_of(fused, device).replay, steps, device)
    t_st = time_device(lambda: ops.row_stats(x, ln.eps, *stats), steps, device)
    return {"tokens": t, "d": cfg.d, "F": f, "layernorm_then_up_gate_us": t_un * 1e6, "folded_us": t_fu * 1e6,
            "row_stats_us": t_st * 1e6, "speedup": t_un / t_fu}


def joint_cfg1(device, steps: int = 10) -> dict:
    """The joint consumer on the cfg1 layer shape (T=32768, d=512, F=2048, fp16; h from
    up_gate at 10 % element density, attention context z ~ N(0,1), residual x):
    out = round(round(round(h W2^T + b2) + round(z Wo^T + bo)) + x) as one kernel,
    against our down projection followed by PyTorch's output projection and adds,
    and against stock PyTorch for all of it; each captured as a CUDA graph, the three timed
    in turn twice (after three untimed replays each), each keeping its faster pass."""
    import torch
    import torch.nn.functional as fn

    from sparsity_spillover_b200 import ops, workloads

    cfg = workloads.CONFIGS["cfg1"]
    layer = workloads.make_weights(cfg, device)[0]
    x = workloads.make_input(cfg, device)
    t, d, f = x.shape[0], cfg.d, cfg.F
    zc = torch.empty(t, f, dtype=cfg.dtype, device=device)
    ops.up_gate(x, layer.w_in, layer.b_in, {"operator": "identity"}, z_out=zc)
    gate = {"operator": "one_sided_threshold", "kappa": workloads.quantile_threshold(zc, DENSITY)}
    del zc
    h, bits = ops.up_gate(x, layer.w_in, layer.b_in, gate)
    g = torch.Generator(device=device).manual_seed(77)
    z = torch.randn(t, d, generator=g, device=device).to(cfg.dtype)
    wo = (torch.randn(d, d, generator=g, device=device) * 0.02).to(cfg.dtype)
    bo = (torch.randn(d, generator=g, device=device) * 0.02).to(cfg.dtype)
    out, y, out_split = (torch.empty(t, d, dtype=cfg.dtype, device=device) for _ in range(3))

    def fused():
        ops.joint(h, bits, z, layer.w_out, layer.b_out, wo, bo, x, out=out)

    def split():
        ops.down_sparse(h, bits, layer.w_out, layer.b_out, y=y)
        torch.add(torch.add(y, fn.linear(z, wo, bo)), x, out=out_split)

    def stock():
        return torch.add(torch.add(fn.linear(h, layer.w_out, layer.b_out), fn.linear(z, wo, bo)), x)

    # Each variant as its own graph; the three are timed in turn, twice, and each keeps its
    # faster pass (the first replays after a capture run slower on some boxes).
    graphs = {name: graph_of(f_, device) for name, f_ in (("fused", fused), ("split", split), ("stock", stock))}
    times = {name: float("inf") for name in graphs}
    for _ in range(2):
        for name, g_ in graphs.items():
            for _ in range(3):
                g_.replay()
            times[name] = min(times[name], time_device(g_.replay, steps, device))
    ref = stock()
    torch.cuda.synchronize(device)
    err = float((out.double() - ref.double()).abs().max() / ref.double().abs().max())
    flop = 2.0 * t * f * d + 2.0 * t * d * d
    tflops = flop / times["fused"] / 1e12
    return {"tokens": t, "d": d, "F": f, "density": DENSITY, "fused_us": times["fused"] * 1e6,
            "down_sparse_plus_torch_us": times["split"] * 1e6, "stock_pytorch_us": times["stock"] * 1e6,
            "speedup_vs_split": times["split"] / times["fused"], "speedup_vs_stock": times["stock"] / times["fused"],
            "executed_tflops": tflops, "max_rel_diff_vs_stock_pytorch": err}


def dff_split_measure(device, world: int, rank: int, layers: int = 4, steps: int = 3) -> dict:
    """410M shape, `layers` layers: d_ff split over the ranks, with the reduce-scatter and the
    next layer's all-gather either as NCCL collectives or fused into the kernels (P2P over
    NVLink), against token sharding of the same per-rank token count (no collective)."""
    import torch
    import torch.distributed as dist

    from sparsity_spillover_b200 import dist as sdist
    from sparsity_spillover_b200 import ops, workloads

    cfg = workloads.CONFIGS["cfg3"]
    full = workloads.make_weights(cfg, device)[:layers]
    gate = {"operator": "one_sided_threshold", "kappa": 0.58}
    t_rank = cfg.tokens
    x_all = workloads.make_input(cfg, device, tokens=t_rank * world)  # the same token block on every rank
    split = [sdist.DffSplitMLP.from_full(L.w_in, L.b_in, L.w_out, L.b_out, gate, world, rank) for L in full]

    def run_split():
        return sdist.dff_split_forward(split, x_all)

    x_mine = x_all[rank * t_rank:(rank + 1) * t_rank].contiguous()
    h = torch.empty(t_rank, cfg.F, dtype=cfg.dtype, device=device)
    bits = torch.empty(ops.tile_bits_size(t_rank, cfg.F), dtype=torch.int32, device=device)
    bufs = [torch.empty_like(x_mine) for _ in range(2)]

    def run_tokens():
        cur = x_mine
        for i, L in enumerate(full):
            cur = ops.mlp_forward(cur, L.w_in, L.b_in, L.w_out, L.b_out, gate, residual=cur, h=h, bits=bits,
                                  y=bufs[i % 2])
        return cur

    # The fused split in both forms: partials stored into peers' receive buffers, and the
    # reduction + broadcast through NVSwitch multicast (when the system offers it).
    fused_peer = sdist.FusedDffSplit(split, t_rank * world, multicast=False)
    runs = [("dff_split", run_split), ("dff_split_fused_peer", lambda: fused_peer.forward(x_all, check=False))]
    fused_mc = None
    if sdist.multicast_available(device):
        fused_mc = sdist.FusedDffSplit(split, t_rank * world, multicast=True)
        runs.append(("dff_split_fused_multicast", lambda: fused_mc.forward(x_all, check=False)))
    # the product's default form in token slices on their own streams, so that one slice's
    # reduction over NVLink overlaps the next slice's projections
    pipes = {n: sdist.PipelinedDffSplit(split, t_rank * world, parts=n) for n in (2, 4)}
    for n, pipe in pipes.items():
        runs.append((f"dff_split_pipelined{n}", lambda pipe=pipe: pipe.forward(x_all, check=False)))
    # the exchange alone and the projections alone, which bound the pipelined forms
    form = fused_mc if fused_mc is not None and world >= sdist.FusedDffSplit.MULTICAST_MIN_WORLD else fused_peer

    def exchanges_only():
        for i in range(layers):
            form.layer_exchange(i)

    def projections_only():
        for i in range(layers):
            form.layer_gemms(i)
    runs.append(("token_sharded", run_tokens))
    out = {}
    for name, fn in runs + [("dff_split_exchanges_only", exchanges_only),
                            ("dff_split_projections_only", projections_only)]:
        fn()
        dist.barrier(device_ids=[device.index])
        t = max_over_ranks(time_device(fn, steps, device), world, device)
        if name.endswith("_only"):
            out[f"{name}_ms_per_step"] = t * 1e3
            continue
        out[f"{name}_tokens_per_s"] = world * t_rank / t
        out[f"{name}_ms_per_step"] = t * 1e3
    # the product's default choice at this world size (FusedDffSplit(multicast=None))
    chosen = "multicast" if fused_mc is not None and world >= sdist.FusedDffSplit.MULTICAST_MIN_WORLD else "peer"
    out["dff_split_fused_tokens_per_s"] = out[f"dff_split_fused_{chosen}_tokens_per_s"]
    out["dff_split_fused_ms_per_step"] = out[f"dff_split_fused_{chosen}_ms_per_step"]
    out["dff_split_fused_form"] = chosen
    out.update(layers=layers, tokens_per_rank=t_rank, world=world,
               collective_bytes_per_layer=2 * (world - 1) * t_rank * cfg.d * 2)
    out["parity"] = dff_split_parity(runs, run_tokens, world, device, split, full, x_all, t_rank, rank)
    return out


def dff_split_parity(runs, run_tokens, world: int, device, split, full, x_all, t_rank: int, rank: int) -> dict:
    """Parity of the d_ff split on this rank's token block, max over ranks.

    Per layer (2e-3 in fp16): one layer of each form (NCCL, fused peer,
    fused multicast) against ops.mlp_forward of the same layer on this rank's tokens on one
    GPU, max|y - y_ref| / max|y_ref|.  Chained: the whole `layers`-deep run of each form
    against the one-GPU chain; there the forms' different rounding of partial sums moves
    layer 2's z by an ulp here and there, and a gate decision at kappa then flips, so the
    chained figure grows with depth and is reported, not held to the bar."""
    import torch
    import torch.distributed as dist

    from sparsity_spillover_b200 import dist as sdist
    from sparsity_spillover_b200 import ops

    def rel(y, ref):
        ref64 = ref.double()
        return float((y.double() - ref64).abs().max()) / max(float(ref64.abs().max()), 1e-30)

    # one layer
    x_mine = x_all[rank * t_rank:(rank + 1) * t_rank].contiguous()
    L0 = full[0]
    ref1 = ops.mlp_forward(x_mine, L0.w_in, L0.b_in, L0.w_out, L0.b_out, split[0].gate, residual=x_mine)
    one = [("dff_split", lambda: sdist.dff_split_forward(split[:1], x_all))]
    peer1 = sdist.FusedDffSplit(split[:1], t_rank * world, multicast=False)
    one.append(("dff_split_fused_peer", lambda: peer1.forward(x_all, check=False)))
    if sdist.multicast_available(device):
        mc1 = sdist.FusedDffSplit(split[:1], t_rank * world, multicast=True)
        one.append(("dff_split_fused_multicast", lambda: mc1.forward(x_all, check=False)))
    parts = 4
    pipe1 = sdist.PipelinedDffSplit(split[:1], t_rank * world, parts=parts)

    def run_pipe1():
        # rank r's blocks of the slices, against the same tokens' rows of ref over all tokens
        return torch.cat(pipe1.forward(x_all, check=False))

    sub, span = t_rank // parts, t_rank * world // parts
    ref1_pipe = torch.cat([ops.mlp_forward(xs, L0.w_in, L0.b_in, L0.w_out, L0.b_out, split[0].gate, residual=xs)
                           for xs in (x_all[p * span + rank * sub:p * span + (rank + 1) * sub].contiguous()
                                      for p in range(parts))])
    errs, names = [], []
    for name, fn in one:
        y = fn()
        torch.cuda.synchronize(device)
        errs.append(rel(y, ref1))
        names.append(name)
    y = run_pipe1()
    torch.cuda.synchronize(device)
    errs.append(rel(y, ref1_pipe))
    names.append(f"dff_split_pipelined{parts}")
    # the chain
    ref = run_tokens().clone()
    chained = []
    for name, fn in runs:
        if name == "token_sharded" or name.startswith("dff_split_pipelined"):
            continue
        y = fn()
        torch.cuda.synchronize(device)
        chained.append(rel(y, ref))
    status = ops.device_status(device.index)
    vec = torch.tensor(errs + chained + [float(status)], dtype=torch.float64, device=device)
    dist.all_reduce(vec, op=dist.ReduceOp.MAX)
    vals = vec.cpu().tolist()
    res = {f"{n}_max_rel_err": vals[i] for i, n in enumerate(names)}
    chained_names = [n for n in names if not n.startswith("dff_split_pipelined")]
    res.update({f"{n}_chained_max_rel_err": vals[len(names) + i] for i, n in enumerate(chained_names)})
    res["reference"] = ("one layer: ops.mlp_forward of that layer on this rank's tokens on one GPU (fp16); chained: "
                        "the one-GPU chain of all the layers")
    res["tolerance"] = 2e-3
    res["ok"] = all(v <= 2e-3 for v in vals[:len(names)]) and vals[-1] == 0
    res["device_status_max"] = int(vals[-1])
    return res


def cfg0_block(device, reps: int = 64, steps: int = 10) -> dict:
    """cfg0, the Pythia-14M MLP block (T=4096, d=128, F=512, one-sided gate at 10 % density),
    on the exact seeded tensors of the reference's CPU case: on the GPU in fp16 as one CUDA
    graph of `reps` back-to-back forwards (the shape is HBM- and launch-bound; the graph
    amortises launches), against stock PyTorch captured the same way; and the reference's
    CPU path (the fp32 oracle restatement) on the same tensors with every host thread."""
    import torch

    from oracle import gates as og
    from oracle import mlp as omlp
    from sparsity_spillover_b200 import ops, workloads

    cfg = workloads.CONFIGS["cfg0"]
    L = workloads.make_weights(cfg, "cpu", dtype=torch.float32)[0]
    x32 = workloads.make_input(cfg, "cpu", dtype=torch.float32)
    t, d, f = cfg.tokens, cfg.d, cfg.F
    # CPU arm: fp32, the reference's kthvalue threshold of z
    with torch.inference_mode():
        z32 = omlp.linear(x32, L.w_in, L.b_in)
        k32 = max(0.0, og.kthvalue_threshold(z32, cfg.density))
        omlp.mlp_forward_fp32(x32, L.w_in, L.b_in, L.w_out, L.b_out, og.ONE_SIDED, k32)
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < 5.0 or n < 3:
            omlp.mlp_forward_fp32(x32, L.w_in, L.b_in, L.w_out, L.b_out, og.ONE_SIDED, k32)
            n += 1
        cpu_s = (time.perf_counter() - t0) / n
    # GPU arm: the same tensors in fp16
    x = x32.half().to(device)
    w_in, b_in, w_out, b_out = (v.half().to(device) for v in (L.w_in, L.b_in, L.w_out, L.b_out))
    z = torch.empty(t, f, dtype=torch.float16, device=device)
    ops.up_gate(x, w_in, b_in, {"operator": "identity"}, z_out=z)
    gate = {"operator": "one_sided_threshold", "kappa": workloads.quantile_threshold(z, cfg.density)}
    h = torch.empty(t, f, dtype=torch.float16, device=device)
    bits = torch.empty(ops.tile_bits_size(t, f), dtype=torch.int32, device=device)
    y = torch.empty(t, d, dtype=torch.float16, device=device)

    def ours():
        for _ in range(reps):
            ops.mlp_forward(x, w_in, b_in, w_out, b_out, gate, h=h, bits=bits, y=y)

    def stock():
        for _ in range(reps):
            zz = torch.nn.functional.linear(x, w_in, b_in)
            torch.nn.functional.linear(zz.masked_fill(zz < gate["kappa"], 0.0), w_out, b_out)

    t_ours = time_device(graph_of(ours, device).replay, steps, device) / reps
    t_stock = time_device(graph_of(stock, device).replay, steps, device) / reps
    density = float((h != 0).float().mean())
    nbytes = 2.0 * (t * d + f * d + f + 2 * t * f + f * d + d + t * d) + t * f / 8192.0
    return {"tokens": t, "d": d, "F": f, "density_measured": round(density, 4),
            "gpu_us_per_forward": t_ours * 1e6, "gpu_tokens_per_s": t / t_ours,
            "stock_pytorch_us_per_forward": t_stock * 1e6, "speedup_vs_stock": t_stock / t_ours,
            "gpu_algorithmic_gbs": nbytes / t_ours / 1e9,
            "gpu_execution": f"CUDA graph of {reps} forwards (up_gate + down_sparse), fp16",
            "cpu_tokens_per_s": t / cpu_s, "cpu_ms_per_forward": cpu_s * 1e3,
            "cpu_threads": torch.get_num_threads(), "cpu_kind": "port (fp32 oracle restatement)",
            "gpu_over_cpu": cpu_s / t_ours}


def host_link(device, nbytes: int, world: int, reps: int = 5) -> dict:
    """Copy-only probe of this rank's host link with the e2e step's byte count: pinned host ->
    device, device -> pinned host, and both at once on two streams (GB/s, each the max time over
    ranks, all ranks copying at the same time)."""
    import torch

    host_in = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    host_out = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    dev_a = torch.empty(nbytes, dtype=torch.uint8, device=device)
    dev_b = torch.empty(nbytes, dtype=torch.uint8, device=device)
    s1, s2 = torch.cuda.Stream(device), torch.cuda.Stream(device)

    def timed(fn) -> float:
        fn()
        torch.cuda.synchronize(device)
        barrier(world, device)
        t0 = time.perf_counter()
        for _ in range(reps):
            fn()
        torch.cuda.synchronize(device)
        dt = (time.perf_counter() - t0) / reps
        return max_over_ranks(dt, world, device)

    def h2d():
        with torch.cuda.stream(s1):
            dev_a.copy_(host_in, non_blocking=True)

    def d2h():
        with torch.cuda.stream(s2):
            host_out.copy_(dev_b, non_blocking=True)

    def both():
        h2d()
        d2h()

    t_in, t_out, t_both = timed(h2d), timed(d2h), timed(both)
    return {"bytes_each_way": nbytes, "h2d_gbs": nbytes / t_in / 1e9, "d2h_gbs": nbytes / t_out / 1e9,
            "concurrent_gbs_each_way": nbytes / t_both / 1e9, "concurrent_ms": t_both * 1e3,
            "timing": "host clock around synchronised copies, max over ranks"}


def summarize(line: dict) -> dict:
    """The per-config figures in a few short keys (kept at the end of the JSON line)."""
    out: dict = {}

    def r(v, n=3):
        return None if v is None else round(float(v), n)

    sweep = line.get("density_sweep")
    if isinstance(sweep, list):
        out["density_sweep_mtok_s"] = {str(x["density_target"]): r(x["tokens_per_s"] / 1e6, 2) for x in sweep}
        out["density_sweep_speedup_vs_rho1"] = {str(x["density_target"]): r(x["speedup_vs_ours_at_100pct"])
                                                for x in sweep}
        out["density_sweep_speedup_vs_stock"] = {str(x["density_target"]): r(x["speedup_vs_dense_pytorch"])
                                                 for x in sweep}
    c2 = line.get("tile_structured_cfg2")
    if isinstance(c2, list):
        out["cfg2_us"] = {f"d{x['d']}_p{x['p']}": [r(x["down_fine_us"], 1), r(x["down_coarse_us"], 1),
                                                   r(x["cublas_us"], 1), r(x["skipped_k16_fraction_fine"])]
                          for x in c2}
        out["cfg2_us_fields"] = ["fine", "coarse", "cublas", "skipped_k16_fraction_fine"]
    ct = line.get("corner_tiles_cfg1")
    if isinstance(ct, list):
        out["corner_tiles_us"] = {f"p{x['p']}": [r(x["dense_us"], 1), r(x["fine_us"], 1), r(x["compact_fine_us"], 1),
                                                 r(x["cublas_us"], 1), r(x["compact_fine_skipped_k16_fraction"])]
                                  for x in ct}
        out["corner_tiles_us_fields"] = ["dense", "fine", "compact_fine", "cublas", "skipped_k16_fraction_compact_fine"]
    c3 = line.get("pythia410m_cfg3")
    if isinstance(c3, dict) and "tokens_per_s" in c3:
        out["cfg3_mtok_s"] = r(c3["tokens_per_s"] / 1e6)
        out["cfg3_executed_tflops"] = r(c3["executed_tflops"], 1)
        out["cfg3_speedup_vs_stock"] = r(c3["speedup_vs_dense_pytorch"])
    j = line.get("joint_cfg1")
    if isinstance(j, dict) and "fused_us" in j:
        out["joint_us"] = {"fused": r(j["fused_us"], 1), "stock": r(j["stock_pytorch_us"], 1),
                           "speedup": r(j["speedup_vs_stock"])}
    hd = line.get("vocab_head_cfg4")
    if isinstance(hd, list):
        out["head_speedup_vs_cublas"] = {
            (f"d{x['d']}_k{x['kappa']}" if x.get("mode") else f"d{x['d']}_n{x['active_fraction']}"):
                r(x["speedup_vs_cublas"]) for x in hd}
        dense = {f"d{x['d']}": r(x["cublas_us"] / x["dense_us"]) for x in hd if "dense_us" in x}
        out["head_dense_speedup_vs_cublas"] = dense
    c0 = line.get("cfg0_block")
    if isinstance(c0, dict) and "gpu_tokens_per_s" in c0:
        out["cfg0"] = {"gpu_mtok_s": r(c0["gpu_tokens_per_s"] / 1e6, 1), "cpu_ktok_s": r(c0["cpu_tokens_per_s"] / 1e3, 1),
                       "speedup_vs_stock": r(c0["speedup_vs_stock"])}
    hl = line.get("host_link")
    if isinstance(hl, dict) and "h2d_gbs" in hl:
        out["host_link_gbs"] = [r(hl["h2d_gbs"], 1), r(hl["d2h_gbs"], 1), r(hl["concurrent_gbs_each_way"], 1)]
    ds = line.get("dff_split_cfg3")
    if isinstance(ds, dict) and "parity" in ds:
        def form(k):
            k = k[:-len("_tokens_per_s")]
            return k[len("dff_split"):].strip("_") or "nccl" if k.startswith("dff_split") else k

        out["dff_split_mtok_s"] = {form(k): r(v / 1e6, 2) for k, v in ds.items() if k.endswith("_tokens_per_s")}
        nccl = ds.get("dff_split_tokens_per_s")
        best = max((v, k) for k, v in ds.items() if k.startswith("dff_split_") and k.endswith("_tokens_per_s"))
        if nccl:
            out["dff_split_best_vs_nccl"] = [form(best[1]), r(best[0] / nccl)]
        out["dff_split_parity"] = {k: (round(v, 6) if isinstance(v, float) else v)
                                   for k, v in ds["parity"].items() if k != "reference"}
    out["value_mtok_s"] = r(line["value"] / 1e6, 2)
    out["e2e_mtok_s"] = r(line["e2e"]["value"] / 1e6, 2)
    out["roofline_frac"] = r(line["roofline"]["frac"])
    return out


def _extra(fn, *args):
    """A secondary measurement: its failure is recorded in the JSON line, never fatal to it."""
    try:
        return fn(*args)
    except Exception as exc:  # noqa: BLE001 - reported, not hidden
        return {"error": f"{type(exc).__name__}: {exc}"[:300]}


def time_device(fn, steps: int, device) -> float:
    import torch

    fn()  # warm-up (first-call library heuristics, lazy set-up)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(device)
    start.record()
    for _ in range(steps):
        fn()
    stop.record()
    torch.cuda.synchronize(device)
    return start.elapsed_time(stop) / 1e3 / steps


def cpu_baseline(cfg, density: float, seconds: float = 12.0) -> dict:
    """The reference's CPU path (oracle restatement, fp32) on a bounded token sample."""
    import torch

    from oracle import gates as og
    from oracle import mlp as omlp
    from sparsity_spillover_b200 import workloads

    threads = torch.get_num_threads()
    sample = 2048
    layers = workloads.make_weights(cfg, "cpu", dtype=torch.float32)
    x0 = workloads.make_input(cfg, "cpu", tokens=sample, dtype=torch.float32)
    kappas = []
    x = x0
    with torch.inference_mode():
        for L in layers:
            z = omlp.linear(x, L.w_in, L.b_in)
            k = max(0.0, og.kthvalue_threshold(z, density))
            kappas.append(k)
            x = omlp.mlp_forward_fp32(x, L.w_in, L.b_in, L.w_out, L.b_out, og.ONE_SIDED, k)[2] + x

        def run():
            xx = x0
            for L, k in zip(layers, kappas):
                xx = omlp.mlp_forward_fp32(xx, L.w_in, L.b_in, L.w_out, L.b_out, og.ONE_SIDED, k)[2] + xx
            return xx

        run()
        reps, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < seconds or reps < 2:
            run()
            reps += 1
        dt = (time.perf_counter() - t0) / reps
    return {"value": sample / dt, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{sample} tokens x {cfg.layers} layers fp32 (GPTNeoXMLP + FixedOneSidedThreshold restated, "
                      f"torch CPU), {reps} reps in {dt * reps:.1f}s",
            "cpu": _cpu_model(), "os_cpu_count": os.cpu_count()}


def _cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_ours(args):
    import torch

    world, rank, local = dist_setup("nccl")
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    from sparsity_spillover_b200 import ops

    with torch.inference_mode():
        stack = Stack(device, rank, DENSITY)
        cfg = stack.cfg
        t, d, f, nl = cfg.tokens, cfg.d, cfg.F, cfg.layers
        for _ in range(args.warmup):
            stack.step()
        torch.cuda.synchronize(device)

        # ---- timed region 1 (value): K steps, each the 6-layer forward replayed as one CUDA graph
        graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(side):
            with torch.cuda.graph(graph, stream=side):
                stack.step()
        torch.cuda.current_stream(device).wait_stream(side)
        for _ in range(args.warmup):
            graph.replay()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        sampler = ClockSampler(list(range(world)) if world > 1 else [local]) if rank == 0 else None
        if sampler:
            sampler.start()
            time.sleep(0.3)
        barrier(world, device)
        torch.cuda.synchronize(device)
        start.record()
        for _ in range(args.steps):
            graph.replay()
        stop.record()
        torch.cuda.synchronize(device)
        barrier(world, device)
        elapsed = start.elapsed_time(stop) / 1e3
        t_step = max_over_ranks(elapsed / args.steps, world, device)

        # ---- timed region 2 (roofline): K eager steps with CUDA events around every kernel,
        # recorded on the stream the kernels are launched on
        ev = [[[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(nl)] for _ in range(args.steps)]
        barrier(world, device)
        torch.cuda.synchronize(device)
        for k in range(args.steps):
            stack.step(events=ev[k])
        torch.cuda.synchronize(device)
        barrier(world, device)
        clocks = sampler.stop() if sampler else None
        t_up = statistics.fmean(e[0].elapsed_time(e[1]) for step in ev for e in step) / 1e3
        t_dn = statistics.fmean(e[1].elapsed_time(e[2]) for step in ev for e in step) / 1e3
        t_up = max_over_ranks(t_up, world, device)
        t_dn = max_over_ranks(t_dn, world, device)
        del graph

        # ---- end to end through the public API: pinned host x -> device -> 6 layers -> host y
        from sparsity_spillover_b200 import pipeline

        mstack = pipeline.MLPStack([pipeline.Layer(L.w_in, L.b_in, L.w_out, L.b_out, g)
                                    for L, g in zip(stack.layers, stack.gates)])
        # Every step copies its batch host->device and its result device->host; batch i+1's
        # H2D and batch i-1's D2H overlap batch i's compute (double-buffered slots).
        x_host = stack.x0.cpu().pin_memory()
        y_hosts = [torch.empty_like(x_host).pin_memory() for _ in range(2)]
        mstack.stream_host([x_host] * args.warmup, [y_hosts[i % 2] for i in range(args.warmup)])
        torch.cuda.synchronize(device)
        e2e_ok = bool(torch.equal(y_hosts[0], stack.step().cpu()))
        barrier(world, device)
        start_e, stop_e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(device)
        start_e.record()
        mstack.stream_host([x_host] * args.steps, [y_hosts[i % 2] for i in range(args.steps)])
        stop_e.record()
        torch.cuda.synchronize(device)
        t_e2e = max_over_ranks(start_e.elapsed_time(stop_e) / 1e3 / args.steps, world, device)
        link = _extra(host_link, device, t * d * 2, world)

        # ---- the same forward as stock PyTorch on CUDA (cuBLAS + masked_fill), for the ratio
        # (captured as a CUDA graph too, so both sides run without host launch gaps)
        for _ in range(2):
            dense_reference_step(stack)
        dgraph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(side):
            with torch.cuda.graph(dgraph, stream=side):
                dense_reference_step(stack)
        torch.cuda.current_stream(device).wait_stream(side)
        dense_ref_t = time_device(dgraph.replay, max(3, args.steps // 2), device)
        del dgraph
        stats = stack.stats.cpu().tolist()
        status = ops.device_status(local)

    p, pk = peaks()
    flop_up = 2.0 * t * d * f
    flop_dn = 2.0 * t * d * f  # random element masks leave every 128x64 K-tile live; dense work is issued
    dom = "up_gate" if t_up >= t_dn else "down_sparse"
    t_dom = t_up if dom == "up_gate" else t_dn
    peak_tf = p["bf16_tflops"]
    achieved = (flop_up if dom == "up_gate" else flop_dn) / t_dom / 1e12
    traffic = NCU_TRAFFIC_BYTES.get(dom)
    # density-scaled algorithmic work of the whole step (f(ormula): L (2Tdf + 2Tdf rho))
    ideal_flop = nl * (2.0 * t * d * f + 2.0 * t * d * f * DENSITY)
    # the matching bytes (2-byte activations and weights): x, W_in, b_in, h written, the live
    # fraction rho_t of h read back, W_out, b_out, y, and the 16x64 bitmap (one bit per 1024 values)
    rho_t = stats[0] / max(1, stats[0] + stats[1])
    ideal_bytes = nl * 2.0 * (t * d + d * f + f + t * f + rho_t * t * f + f * d + d + t * d) + nl * t * f / 8192.0
    t_flop_s, t_byte_s = ideal_flop / (peak_tf * 1e12), ideal_bytes / (p["hbm_gbs"] * 1e9)
    bound_s = max(t_flop_s, t_byte_s)
    value = world * t / t_step
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": t_step * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp16", "data": "synthetic (seeded N(0,1) x, GPT-NeoX init weights)",
        "config": {"workload": WORKLOAD, "tokens_per_gpu": t, "layers": nl, "density_target": DENSITY,
                   "density_measured": stack.density, "parallelism": f"token-sharded x{world}",
                   "l2": "working set per step > L2 (h alone is 134 MB per layer)"},
        "roofline": {"kernel": dom, "bound": "tensor", "achieved": achieved, "peak": peak_tf, "unit": "TFLOP/s",
                     "frac": achieved / peak_tf, "traffic": traffic, "peak_source": f"{pk} bf16_tflops (burst)",
                     "up_gate_us": t_up * 1e6, "down_sparse_us": t_dn * 1e6},
        "density_scaled_roofline": {"algorithmic_tflop_per_step": ideal_flop / 1e12,
                                    "achieved_tflops": ideal_flop / t_step / 1e12,
                                    "frac": ideal_flop / t_step / 1e12 / peak_tf,
                                    "live_k16_fraction": rho_t, "algorithmic_gb_per_step": ideal_bytes / 1e9,
                                    "achieved_gbs": ideal_bytes / t_step / 1e9,
                                    "frac_hbm": ideal_bytes / t_step / 1e9 / p["hbm_gbs"],
                                    "time_bound_us": bound_s * 1e6, "bound": "tensor" if t_flop_s >= t_byte_s else "hbm",
                                    "step_over_bound": t_step / bound_s},
        "skip_stats_calibration": {"issued_k16": stats[0], "skipped_k16": stats[1]},
        "dense_pytorch_cuda": {"tokens_per_s": t / dense_ref_t, "speedup": dense_ref_t / (t_step)},
        "e2e": {"value": world * t / t_e2e, "unit": "tokens/s", "h2d_bytes_per_step": t * d * 2,
                "d2h_bytes_per_step": t * d * 2, "pipelining": "batches: H2D(i+1) and D2H(i-1) overlap compute(i)",
                "matches_device_forward": e2e_ok, "ms_per_step": t_e2e * 1e3},
        "gpu_launches": args.steps * nl * 2,
        "execution": "value: CUDA-graph replay of the 6-layer step (12 kernels per step: up_gate and "
                     "down_sparse per layer, chained by programmatic dependent launch); "
                     "roofline: eager steps with per-kernel CUDA events",
        "clocks": clocks,
        "device_status": status,
        "host_link": link,
    }
    if world > 1 and not args.no_extras:
        line["dff_split_cfg3"] = _extra(dff_split_measure, device, world, rank)
    if world == 1 and not args.no_extras:
        import torch

        with torch.inference_mode():
            line["density_sweep"] = _extra(density_sweep, device)
            line["paired_protocol_cfg1"] = _extra(paired_cfg1, device)
            line["tile_structured_cfg2"] = _extra(tile_structured, device)
            line["pythia410m_cfg3"] = _extra(cfg3_410m, device)
            line["vocab_head_cfg4"] = _extra(head_bench, device)
            line["joint_cfg1"] = _extra(joint_cfg1, device)
            line["layernorm_fold_cfg1"] = _extra(layernorm_fold_cfg1, device)
            line["cfg0_block"] = _extra(cfg0_block, device)
            line["corner_tiles_cfg1"] = _extra(corner_tiles_cfg1, device)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(cfg, DENSITY)
    if world > 1:
        import torch.distributed as dist

        dist.barrier(device_ids=[device.index])
        dist.destroy_process_group()
    if rank == 0:
        line["summary"] = summarize(line)  # last key: survives a truncated tail of the output
        print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- reference arm
def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import torch

    from sparsity_spillover_b200 import workloads

    cfg = workloads.CONFIGS["cfg1"]
    torch.set_num_threads(os.cpu_count() or 1)
    # Each step: the 6-layer fp32 CPU forward of a bounded token sample.
    per_step_seconds = max(1.0, 60.0 / max(1, args.steps + args.warmup))
    base = cpu_baseline(cfg, DENSITY, seconds=per_step_seconds)
    value = base["value"]
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 2048 / value * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp32", "data": "synthetic (seeded N(0,1) x, GPT-NeoX init weights)",
        "config": {"workload": WORKLOAD, "tokens_per_gpu": cfg.tokens, "layers": cfg.layers,
                   "density_target": DENSITY, "parallelism": "host cores (the reference's CPU path, oracle port)",
                   "sample": "each step times a 2048-token sample of this workload"},
        "impl": "reference",
        "cpu_baseline": {"kind": base["kind"], "cores": base["cores"], "sample": base["sample"], "value": value,
                         "unit": "tokens/s"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="skip the per-config sweeps (density, cfg2, cfg3, cfg4)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
