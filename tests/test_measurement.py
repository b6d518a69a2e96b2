"""The paired, rotating-input timing protocol (sparsity_spillover_b200.measurement) against
golden outputs of the reference harness's own functions
(runs/025-…/measurement.py:26-97, fixtures from tests/golden/make_golden.py)."""
from __future__ import annotations

import math
from pathlib import Path

import numpy as np
import pytest

from sparsity_spillover_b200 import measurement

GOLDEN = np.load(Path(__file__).parent / "golden" / "measurement.npz")
SCHEDULE_CASES = [(1, 1, ("native",), 0), (3, 2, ("native", "fused", "sparse"), 7),
                  (4, 3, ("dense_pytorch", "ours_rho100", "ours_rho10"), 2026), (5, 2, ("a", "b"), 123456789)]


@pytest.mark.parametrize("case", range(len(SCHEDULE_CASES)))
def test_schedule_matches_reference(case):
    count, passes, modes, seed = SCHEDULE_CASES[case]
    rows = measurement.paired_schedule(count, passes, list(modes), seed)
    got = np.array([[rep, idx] + [modes.index(m) for m in order] for rep, idx, order in rows])
    np.testing.assert_array_equal(got, GOLDEN[f"schedule{case}"])
    # every (pass, input) once, every mode once per block
    assert sorted((r, i) for r, i, _ in rows) == [(r, i) for r in range(passes) for i in range(count)]
    assert all(sorted(o) == sorted(modes) for _, _, o in rows)


@pytest.mark.parametrize("args", [(0, 1, ("a",), 0), (1, 0, ("a",), 0), (1, 1, (), 0), (1, 1, ("a", "a"), 0)])
def test_schedule_rejects_invalid(args):
    count, passes, modes, seed = args
    with pytest.raises(ValueError):
        measurement.paired_schedule(count, passes, list(modes), seed)


def _fixed_samples():
    modes = ("native", "a", "b")
    host = iter(GOLDEN["summary_host_ms"].tolist())
    return [{"repeat": rep, "input_index": idx, "mode": m, "host_ms": next(host), "cuda_ms": None}
            for rep in range(2) for idx in range(3) for m in modes], modes


def test_summary_matches_reference():
    samples, modes = _fixed_samples()
    summary = measurement.timing_summary(samples, reference="native", tokens_per_call=1000)
    np.testing.assert_allclose([summary[m]["median_host_ms"] for m in modes], GOLDEN["summary_median"], rtol=0, atol=0)
    np.testing.assert_allclose([summary[m]["paired_geomean_speedup"] for m in modes], GOLDEN["summary_geomean"],
                               rtol=1e-15)
    assert summary["native"]["paired_geomean_speedup"] == 1.0
    assert summary["a"]["input_tokens_per_second"] == pytest.approx(1000 / (summary["a"]["median_host_ms"] / 1e3))


def test_summary_rejects_unmatched_and_invalid():
    samples, _ = _fixed_samples()
    with pytest.raises(ValueError):
        measurement.timing_summary(samples[:-1], reference="native")  # mode b lacks one (pass, input) key
    bad = [dict(s) for s in samples]
    bad[1]["host_ms"] = 0.0
    with pytest.raises(ValueError):
        measurement.timing_summary(bad, reference="native")
    with pytest.raises(ValueError):
        measurement.timing_summary(samples, reference="missing")


def test_paired_timing_walks_the_schedule_on_cpu():
    calls = []
    state = {"mode": None}

    def set_mode(m):
        state["mode"] = m

    def forward(x):
        calls.append((state["mode"], x))
        return x

    modes = ["native", "fast"]
    samples = measurement.paired_timing(forward, set_mode, [10, 11, 12], modes=modes, passes=2, warmups=2, seed=5,
                                        cuda=False)
    assert calls[:4] == [("native", 10), ("native", 11), ("fast", 10), ("fast", 11)]  # warm-ups per mode first
    timed = calls[4:]
    sched = measurement.paired_schedule(3, 2, modes, 5)
    assert timed == [(m, 10 + idx) for _, idx, order in sched for m in order]
    assert len(samples) == 12 and all(s["cuda_ms"] is None and s["host_ms"] >= 0 for s in samples)
    summary = measurement.timing_summary([dict(s, host_ms=s["host_ms"] + 1.0) for s in samples], reference="native")
    assert set(summary) == set(modes) and math.isfinite(summary["fast"]["paired_geomean_speedup"])
