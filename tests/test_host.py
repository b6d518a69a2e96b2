"""Host-side logic on CPU: the C ABI loads and exports every declared symbol, the
gate-spec boundary mirrors the reference's validation, workloads and oracle
helpers behave, and nothing computes on CPU tensors (no fallback)."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import bitmap as obit
from oracle import gates as og

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols() -> set[str]:
    text = (ROOT / "include" / "spmlp.h").read_text()
    return set(re.findall(r"^(?:int|int64_t|const char\*)\s+(spmlp_\w+)\(", text, flags=re.M))


def test_library_exports_every_declared_symbol(lib):
    from sparsity_spillover_b200 import _lib

    declared = declared_symbols()
    assert len(declared) >= 12
    for name in declared:
        assert hasattr(lib, name), name
    assert declared == set(_lib.SIGNATURES), declared ^ set(_lib.SIGNATURES)


def test_pure_host_entry_points(lib):
    assert lib.spmlp_version() >= 100
    assert lib.spmlp_tile_bits_words(2048) == 1
    assert lib.spmlp_tile_bits_words(4096) == 2
    assert lib.spmlp_tile_bits_words(64) == 1
    assert lib.spmlp_tile_bits_size(32768, 2048) == 2048
    assert lib.spmlp_tile_bits_size(1000, 320) == 63
    assert lib.spmlp_head_support_words(128) == 1
    assert lib.spmlp_head_support_words(1024) == 2
    assert lib.spmlp_down_tile_tokens(1) == 256 and lib.spmlp_down_tile_tokens(2) == 128
    assert lib.spmlp_last_error() is not None


def test_argument_errors_are_reported_without_a_gpu(lib):
    """Shape and enum checks run before any CUDA call and return negative codes."""
    k = ctypes.c_float(0.5)
    rc = lib.spmlp_up_gate(16, 16, None, 16, 16, None, 64, 100, 512, 0, 2, k, 64, None)
    assert rc == -2 and b"multiple of 64" in lib.spmlp_last_error()
    rc = lib.spmlp_up_gate(16, 16, None, 16, 16, None, 64, 128, 512, 7, 2, k, 64, None)
    assert rc == -1 and b"dtype" in lib.spmlp_last_error()
    rc = lib.spmlp_up_gate(16, 16, None, 16, 16, None, 64, 128, 512, 0, 2, ctypes.c_float(float("nan")), 64, None)
    assert rc == -1 and b"kappa" in lib.spmlp_last_error()
    rc = lib.spmlp_up_gate(17, 16, None, 16, 16, None, 64, 128, 512, 0, 2, k, 64, None)
    assert rc == -3
    rc = lib.spmlp_down_sparse(16, None, 16, None, None, 16, 64, 512, 128, 0, 1, None, None)
    assert rc == -1 and b"tile_bits" in lib.spmlp_last_error()
    rc = lib.spmlp_up_gate(16, 16, None, 16, 16, None, 64, 128, 512, 0, 6, k, 12, None)
    assert rc == -2  # corner gate: T=64 is not a multiple of seq_len=12
    assert lib.spmlp_set_sm_count_target(-1) == -1 and b"sms" in lib.spmlp_last_error()


def test_joint_and_gate_argument_errors_without_a_gpu(lib):
    k = ctypes.c_float(0.5)
    # h, bits, z, w2, b2, wo, bo, residual, out, T, F, d, dtype, mode, stats, stream
    rc = lib.spmlp_joint(16, 16, 16, 16, None, 16, None, None, 16, 64, 512, 128, 0, 7, None, None)
    assert rc == -1 and b"joint mode" in lib.spmlp_last_error()
    rc = lib.spmlp_joint(16, None, 16, 16, None, 16, None, None, 16, 64, 512, 128, 0, 1, None, None)
    assert rc == -1 and b"tile_bits" in lib.spmlp_last_error()
    rc = lib.spmlp_joint(16, None, None, 16, None, 16, None, None, 16, 64, 512, 128, 0, 0, None, None)
    assert rc == -1 and b"non-null" in lib.spmlp_last_error()
    rc = lib.spmlp_joint(16, 16, 16, 16, None, 16, None, None, 16, 64, 512, 100, 0, 1, None, None)
    assert rc == -2
    rc = lib.spmlp_joint(17, 16, 16, 16, None, 16, None, None, 16, 64, 512, 128, 0, 1, None, None)
    assert rc == -3
    # x, out, bits, T, F, dtype, gate_op, kappa, stream
    rc = lib.spmlp_gate(16, 16, None, 64, 512, 0, 1, k, None)
    assert rc == -1 and b"gate" in lib.spmlp_last_error()  # GELU is not an elementwise threshold gate
    rc = lib.spmlp_gate(16, 16, None, 64, 500, 0, 2, k, None)
    assert rc == -2
    rc = lib.spmlp_gate(16, 16, None, 64, 512, 0, 2, ctypes.c_float(-1.0), None)
    assert rc == -1 and b"kappa" in lib.spmlp_last_error()
    rc = lib.spmlp_gate(16, 1024, None, 64, 512, 0, 2, k, None)
    assert rc == -1 and b"overlap" in lib.spmlp_last_error()
    # peer_slots, local_flags, world, epoch, stream
    slots = (ctypes.c_void_p * 2)(16, 24)
    rc = lib.spmlp_peer_barrier(ctypes.cast(slots, ctypes.POINTER(ctypes.c_void_p)), 16, 9, 1, None)
    assert rc == -1 and b"world" in lib.spmlp_last_error()
    rc = lib.spmlp_peer_barrier(ctypes.cast(slots, ctypes.POINTER(ctypes.c_void_p)), 16, 2, 0, None)
    assert rc == -1 and b"epoch" in lib.spmlp_last_error()
    bad = (ctypes.c_void_p * 2)(16, 20)
    rc = lib.spmlp_peer_barrier(ctypes.cast(bad, ctypes.POINTER(ctypes.c_void_p)), 16, 2, 1, None)
    assert rc == -3


def test_joint_consumer_reads_the_reference_gates():
    from types import SimpleNamespace

    from sparsity_spillover_b200 import JointConsumer

    lin2, lino = torch.nn.Linear(512, 128), torch.nn.Linear(128, 128)
    layer = SimpleNamespace(mlp=SimpleNamespace(dense_4h_to_h=lin2, act=FixedOneSidedThreshold(0.25)),
                            attention=SimpleNamespace(dense=lino, z_gate=FixedOneSidedThreshold(0.5)))
    j = JointConsumer(layer)
    assert (j.gh, j.gz, j.th, j.tz) == (True, True, 0.25, 0.5) and j.w2 is lin2 and j.wo is lino
    relu = SimpleNamespace(mlp=SimpleNamespace(dense_4h_to_h=lin2, act=torch.nn.ReLU()),
                           attention=SimpleNamespace(dense=lino))
    j = JointConsumer(relu)
    assert (j.gh, j.gz, j.th) == (True, False, 0.0)
    gelu = SimpleNamespace(mlp=SimpleNamespace(dense_4h_to_h=lin2, act=None),
                           attention=SimpleNamespace(dense=lino, z_gate=FixedSymmetricThreshold(0.1)))
    j = JointConsumer(gelu)
    assert (j.gh, j.gz) == (False, False)  # the reference joint gates only with one-sided z gates
    with pytest.raises(ValueError):
        j(torch.zeros(64, 512), torch.zeros(64, 128), torch.zeros(64, 128))  # CPU tensors: no fallback


def test_folded_layernorm_algebra_on_cpu():
    """rstd * (x (W diag(gamma))^T - mean * s) + c == LN(x) W^T + b (weight preparation only)."""
    from sparsity_spillover_b200 import ops

    g = torch.Generator().manual_seed(4)
    t, d, f = 64, 128, 256
    x = torch.randn(t, d, generator=g, dtype=torch.float64) + 3.0
    gamma, beta = 1 + 0.1 * torch.randn(d, generator=g), 0.1 * torch.randn(d, generator=g)
    w, b = 0.05 * torch.randn(f, d, generator=g), 0.05 * torch.randn(f, generator=g)
    fold = ops.FoldedLayerNorm(gamma, beta, 1e-5, w, b, dtype=torch.float32)
    mean = x.mean(1, keepdim=True)
    rstd = 1.0 / torch.sqrt(x.var(1, unbiased=False, keepdim=True) + 1e-5)
    z = rstd * (x @ fold.w_fold.double().T - mean * fold.s.double()[None, :]) + fold.c.double()[None, :]
    ref = torch.nn.functional.layer_norm(x, (d,), gamma.double(), beta.double(), 1e-5) @ w.double().T + b.double()
    assert torch.allclose(z, ref, rtol=1e-5, atol=1e-5)


def test_ops_refuse_cpu_tensors():
    from sparsity_spillover_b200 import ops

    x = torch.randn(64, 128, dtype=torch.float16)
    w = torch.randn(512, 128, dtype=torch.float16)
    with pytest.raises(ValueError, match="CUDA"):
        ops.up_gate(x, w, None, {"operator": "relu"})
    with pytest.raises(ValueError, match="CUDA"):
        ops.down_sparse(torch.zeros(64, 512, dtype=torch.float16), None, w.T.contiguous(), None, skip=False)
    with pytest.raises(ValueError, match="CUDA"):
        ops.head_sparse(x, w)


# ---------------------------------------------------------------- gate boundary
class FixedOneSidedThreshold(torch.nn.Module):  # same name/attributes as the reference module
    def __init__(self, kappa):
        super().__init__()
        self.kappa = kappa


class FixedSymmetricThreshold(FixedOneSidedThreshold):
    pass


class CornerTileThreshold(torch.nn.Module):
    def __init__(self, kappa, tile_tokens=8, tile_features=16):
        super().__init__()
        self.kappa, self.tile_tokens, self.tile_features = kappa, tile_tokens, tile_features


def test_gate_modules_are_recognised():
    from transformers.activations import ACT2FN

    from sparsity_spillover_b200 import _lib, gates

    assert gates.resolve(FixedOneSidedThreshold(0.25)).op == _lib.GATE_ONE_SIDED
    assert gates.resolve(FixedSymmetricThreshold(0.25)).op == _lib.GATE_SYMMETRIC
    assert gates.resolve(torch.nn.ReLU()).op == _lib.GATE_RELU
    assert gates.resolve(CornerTileThreshold(0.1)).op == _lib.GATE_CORNER
    assert gates.resolve(ACT2FN["gelu"]).op == _lib.GATE_GELU
    assert gates.resolve(None).op == _lib.GATE_GELU
    with pytest.raises(ValueError):
        gates.resolve(torch.nn.GELU(approximate="tanh"))
    with pytest.raises(ValueError):
        gates.resolve(CornerTileThreshold(0.1, 16, 16))  # the h/z corner tile is 8x16


@pytest.mark.parametrize("bad", [
    {"operator": "relu", "kappa": 0.1},
    {"operator": "one_sided_threshold"},
    {"operator": "one_sided_threshold", "kappa": -1.0},
    {"operator": "one_sided_threshold", "kappa": True},
    {"operator": "one_sided_threshold", "kappa": float("nan")},
    {"operator": "symmetric_threshold", "kappa": 0.1, "extra": 1},
    {"operator": "scalar", "kappa": 0.1},
    {"operator": "tile_corner_threshold", "kappa": 0.1, "tile_tokens": 0, "tile_features": 16},
])
def test_gate_spec_validation_mirrors_reference(bad):
    """Same acceptance rules as sites.py:195-214 / _nonnegative_finite and tile_gate.py:48-59."""
    from sparsity_spillover_b200 import gates

    with pytest.raises(ValueError):
        gates.resolve(bad)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("kappa", [0.0, 0.1, 0.3, 1.0 / 3.0, 2.5])
def test_kappa_is_rounded_like_the_reference(dtype, kappa):
    from sparsity_spillover_b200 import gates

    spec = gates.resolve({"operator": "one_sided_threshold", "kappa": kappa})
    assert spec.kappa_for(dtype) == og.round_kappa(kappa, dtype)


def test_sparse_mlp_module_keeps_state_dict_names():
    import transformers
    from transformers.models.gpt_neox.modeling_gpt_neox import GPTNeoXMLP

    from sparsity_spillover_b200 import SparseGPTNeoXMLP, install

    cfg = transformers.GPTNeoXConfig(hidden_size=128, intermediate_size=512, num_hidden_layers=2,
                                     num_attention_heads=4, vocab_size=256)
    mlp = GPTNeoXMLP(cfg)
    mlp.act = FixedOneSidedThreshold(0.2)
    sparse = SparseGPTNeoXMLP.from_mlp(mlp)
    assert set(sparse.state_dict()) == set(mlp.state_dict())
    assert sparse.dense_h_to_4h.weight is mlp.dense_h_to_4h.weight
    model = transformers.GPTNeoXForCausalLM(cfg)
    meta = install(model)
    assert all(isinstance(layer.mlp, SparseGPTNeoXMLP) for layer in model.gpt_neox.layers)
    assert meta["gates"][0] == {"operator": "gelu"}
    with pytest.raises(ValueError):
        with torch.inference_mode():
            sparse(torch.randn(2, 128))  # CPU tensors: no fallback


# ---------------------------------------------------------------- workloads / oracle helpers
def test_tile_structured_workload_has_the_requested_tile_density():
    from sparsity_spillover_b200 import workloads

    h, frac = workloads.tile_structured_h(4096, 1024, 0.2, seed=5, device="cpu")
    assert abs(frac - 0.2) < 0.05
    mask = obit.tile_mask(h, 64, 64)
    assert abs(float(mask.mean()) - frac) < 1e-6
    assert float((h != 0).float().mean()) == pytest.approx(frac, abs=0.01)


def test_zipf_tiles_are_sorted_unique_and_sized():
    from sparsity_spillover_b200 import workloads

    for frac in (0.05, 0.1, 0.25):
        tiles = workloads.zipf_active_tiles(393, frac, seed=3)
        assert len(tiles) == round(frac * 393)
        assert np.all(np.diff(tiles) > 0) and tiles.min() >= 0 and tiles.max() < 393
    assert np.array_equal(workloads.zipf_active_tiles(393, 0.1, 3), workloads.zipf_active_tiles(393, 0.1, 3))


def test_quantile_threshold_hits_density():
    from sparsity_spillover_b200 import workloads

    z = torch.randn(200_000)
    k = workloads.quantile_threshold(z, 0.1)
    assert float((z >= k).float().mean()) == pytest.approx(0.1, abs=0.002)
    assert workloads.quantile_threshold(z, 0.7) == 0.0  # negative thresholds clamp at zero


def test_bitmap_pack_roundtrip_and_skip_counts():
    rng = np.random.default_rng(0)
    mask = rng.random((37, 45)) < 0.3
    words = obit.pack_bits(mask)
    assert words.shape == (37, 2)
    assert np.array_equal(obit.unpack_bits(words, 45), mask)
    h = torch.zeros(256, 128)
    h[0, 0] = 1.0
    h[20, 100] = -0.0  # a negative zero is a zero
    h[40, 127] = 2.0
    m = obit.tile_mask(h)
    assert m.shape == (16, 2) and m.sum() == 2 and m[0, 0] and m[2, 1]
    # First 128-token tile: both 64-feature K-blocks live (4 K16 steps each); second tile: none.
    issued, skipped = obit.skip_counts(m, 128, n_tiles=2)
    assert (issued, skipped) == (2 * 4 * 2, (2 * 8 - 2 * 4) * 2)


def _golden_module():
    import importlib.util

    path = Path(__file__).parent / "golden" / "make_golden.py"
    spec = importlib.util.spec_from_file_location("make_golden_cases", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_head_gate_validation_matches_the_reference():
    """gates.validate_head_gate accepts and rejects exactly what the reference head's
    validate_gate does (golden outcomes from runs/068-…/inference/head.py:20-28)."""
    from sparsity_spillover_b200 import gates

    cases = _golden_module().head_gate_cases()
    expect = np.load(Path(__file__).parent / "golden" / "head_gate.npz")["kappa_or_nan"]
    assert len(cases) == len(expect)
    for spec, want in zip(cases, expect):
        if np.isnan(want):
            with pytest.raises(ValueError, match="corner16x16"):
                gates.validate_head_gate(spec)
        else:
            assert gates.validate_head_gate(spec) == want


def test_install_head_modes_and_checks_on_cpu():
    """The reference head installer's modes, consumer-tile rule and metadata (construction
    only: no kernel runs without a GPU)."""
    import transformers

    from sparsity_spillover_b200 import SparseHead, install_head

    def model():
        cfg = transformers.GPTNeoXConfig(hidden_size=128, intermediate_size=512, num_hidden_layers=1,
                                         num_attention_heads=4, vocab_size=1024)
        m = transformers.GPTNeoXForCausalLM(cfg).eval()
        m.config.head_input_gate = {"operator": "tile_corner_threshold", "kappa": 0.25, "tile_tokens": 16,
                                    "tile_features": 16}
        return m

    with pytest.raises(ValueError):
        install_head(model(), "bogus")
    with pytest.raises(ValueError, match="consumer tile"):
        install_head(model(), "custom_sparse", {"kernel_tile_tokens": 16, "kernel_tile_vocabulary": 64})
    m = model()
    m.config.head_input_gate = {"operator": "tile_corner_threshold", "kappa": 0.25}
    with pytest.raises(ValueError, match="corner16x16"):
        install_head(m, "custom_sparse")
    for mode, skip in (("custom_sparse", True), ("custom_no_skip", False)):
        m = model()
        w = m.embed_out.weight
        meta = install_head(m, mode, {"kernel_tile_tokens": 16, "kernel_tile_vocabulary": 128})
        assert isinstance(m.embed_out, SparseHead) and m.embed_out.weight is w
        assert m.embed_out.kappa == float(torch.tensor(0.25, dtype=torch.float32)) and m.embed_out.skip is skip
        assert meta["mode"] == mode and meta["gate"]["kappa"] == 0.25 and meta["consumer_tile"] == [16, 128, 16]
        with pytest.raises(ValueError, match="already"):
            install_head(m, mode)
    m = model()
    meta = install_head(m, "dense")
    assert m.embed_out.kappa is None and meta["gate"] is None
