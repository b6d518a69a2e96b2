"""The bench line's trailing ``summary`` object (CPU: pure dict arithmetic)."""
from __future__ import annotations

import importlib.util
from pathlib import Path


def _bench():
    spec = importlib.util.spec_from_file_location("bench_for_test", Path(__file__).resolve().parents[1] / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_summary_names_the_dff_split_forms_and_the_best_against_nccl():
    bench = _bench()
    line = {"value": 42.0e6, "e2e": {"value": 38.0e6}, "roofline": {"frac": 0.61},
            "dff_split_cfg3": {"dff_split_tokens_per_s": 26.3e6, "dff_split_fused_peer_tokens_per_s": 16.8e6,
                               "dff_split_fused_multicast_tokens_per_s": 32.3e6,
                               "dff_split_pipelined4_tokens_per_s": 43.3e6, "token_sharded_tokens_per_s": 150.6e6,
                               "dff_split_fused_tokens_per_s": 32.3e6, "dff_split_exchanges_only_ms_per_step": 4.9,
                               "parity": {"ok": True, "tolerance": 2e-3, "reference": "one GPU"}}}
    s = bench.summarize(line)
    assert s["dff_split_mtok_s"] == {"nccl": 26.3, "fused_peer": 16.8, "fused_multicast": 32.3, "pipelined4": 43.3,
                                     "token_sharded": 150.6, "fused": 32.3}
    assert s["dff_split_best_vs_nccl"] == ["pipelined4", round(43.3 / 26.3, 3)]
    assert s["dff_split_parity"] == {"ok": True, "tolerance": 2e-3}
    assert (s["value_mtok_s"], s["e2e_mtok_s"], s["roofline_frac"]) == (42.0, 38.0, 0.61)
    assert list(s)[-1] == "roofline_frac"
