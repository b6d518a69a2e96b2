"""Paired, rotating-input latency protocol of the reference's measurement harness
(runs/025-2026-09-05-pythia-agentic-sparse-kernel-search/measurement.py:26-97).

The protocol, restated:

* ``paired_schedule``: for every pass, the input indices in a shuffled order, and
  for every input index the modes in a shuffled order — one ``random.Random(seed)``
  drives both shuffles in that sequence (measurement.py:26-38), so the same seed
  gives the reference's schedule.
* ``paired_timing``: each mode first runs ``warmups`` untimed calls on its own; then
  the schedule is walked, and every call is bracketed by a device synchronize,
  a host clock and CUDA events on the current stream; the host latency (primary)
  and the CUDA-event latency are both kept (measurement.py:41-77).
* ``timing_summary``: per mode, the median host latency and the geometric mean of
  the per-sample speed-ups ``t_reference / t_mode`` over the samples that share a
  (pass, input) key — every mode must hold exactly the reference mode's keys
  (measurement.py:80-97).

This module is measurement infrastructure for ``bench.py``; it runs any callable
and holds no kernel code.
"""
from __future__ import annotations

import math
import random
import time
from typing import Callable, Iterable, Sequence


def paired_schedule(count: int, passes: int, modes: Sequence[str], seed: int) -> list[tuple[int, int, list[str]]]:
    """[(pass, input_index, mode_order)] for ``passes`` passes over ``count`` inputs."""
    if count <= 0 or passes <= 0 or not modes or len(set(modes)) != len(modes):
        raise ValueError("Invalid paired schedule")
    rng = random.Random(seed)
    schedule = []
    for rep in range(passes):
        order_in = list(range(count))
        rng.shuffle(order_in)
        for idx in order_in:
            order_modes = list(modes)
            rng.shuffle(order_modes)
            schedule.append((rep, idx, order_modes))
    return schedule


def paired_timing(forward: Callable, set_mode: Callable[[str], None], inputs: Sequence, *, modes: Sequence[str],
                  passes: int, warmups: int, seed: int, cuda: bool = True,
                  sample_sink: Callable[[dict], None] = lambda row: None) -> list[dict]:
    """Time ``forward(inputs[i])`` under each mode on the paired schedule.

    ``set_mode(mode)`` selects the implementation (outside the timed region).
    Returns one sample per call: pass, input index, mode, ``host_ms`` (synchronised
    host latency) and ``cuda_ms`` (CUDA events on the current stream, or None)."""
    import torch

    samples: list[dict] = []
    with torch.inference_mode():
        for mode in modes:
            set_mode(mode)
            for i in range(warmups):
                forward(inputs[i % len(inputs)])
            if cuda:
                torch.cuda.synchronize()
        for rep, idx, order in paired_schedule(len(inputs), passes, modes, seed):
            for mode in order:
                set_mode(mode)
                if cuda:
                    torch.cuda.synchronize()
                    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                t0 = time.perf_counter()
                if cuda:
                    ev0.record()
                out = forward(inputs[idx])
                if cuda:
                    ev1.record()
                    ev1.synchronize()
                host_ms = (time.perf_counter() - t0) * 1e3
                row = {"repeat": rep, "input_index": idx, "mode": mode, "host_ms": host_ms,
                       "cuda_ms": ev0.elapsed_time(ev1) if cuda else None}
                samples.append(row)
                sample_sink(row)
                del out
    return samples


def _median(values: Iterable[float]) -> float:
    v = sorted(values)
    return (v[(len(v) - 1) // 2] + v[len(v) // 2]) / 2


def timing_summary(samples: Sequence[dict], reference: str, tokens_per_call: int | None = None) -> dict:
    """Per mode: sample count, median host ms, median CUDA ms (when recorded), the paired
    geometric-mean speed-up over ``reference`` and, given ``tokens_per_call``, the
    input tokens per second at the median host latency."""
    by_mode: dict[str, dict[tuple[int, int], dict]] = {}
    for row in samples:
        by_mode.setdefault(row["mode"], {})[(row["repeat"], row["input_index"])] = row
    if reference not in by_mode:
        raise ValueError(f"no samples of the reference mode {reference!r}")
    ref = by_mode[reference]
    result = {}
    for mode, paired in by_mode.items():
        host = {k: r["host_ms"] for k, r in paired.items()}
        if paired.keys() != ref.keys() or any(not (x > 0 and math.isfinite(x)) for x in host.values()):
            raise ValueError("Unmatched/invalid timing samples")
        logs = [math.log(ref[k]["host_ms"] / x) for k, x in host.items()]
        med = _median(host.values())
        cuda = [r["cuda_ms"] for r in paired.values() if r.get("cuda_ms") is not None]
        result[mode] = {"samples": len(host), "median_host_ms": med,
                        "median_cuda_ms": _median(cuda) if len(cuda) == len(host) else None,
                        "paired_geomean_speedup": math.exp(sum(logs) / len(logs)),
                        "input_tokens_per_second": tokens_per_call / (med / 1e3) if tokens_per_call else None}
    return result
