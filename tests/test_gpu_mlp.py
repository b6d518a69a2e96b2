"""GPU parity of the up-projection + gate + bitmap and the sparse down-projection.

The CUDA path is compared with the CPU oracle (oracle/, pinned to the
reference's own modules by tests/test_oracle_golden.py) on the same seeded
inputs:

* masks and tile bitmaps are bit-exact against the reference gate applied to
  the kernel's own z (parity is defined on the kernel's rounded z);
* z and y are within the north-star tolerance of an fp32 oracle:
  max|err| / max|ref| <= 2e-3 (fp16), 1e-2 (bf16);
* gate decisions that differ from the fp32 oracle's lie within one dtype ulp of kappa;
* the skipping down-projection is bit-identical to the dense one, and its
  issued/skipped counters match the oracle's tile accounting.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import bitmap as obit
from oracle import gates as og
from oracle import mlp as omlp

pytestmark = pytest.mark.gpu

TOL = {torch.float16: 2e-3, torch.bfloat16: 1e-2}
DEV = "cuda"


def _inputs(t, d, f, dtype, seed=0, bias=True):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(t, d, generator=g).to(dtype)
    w_in = (torch.randn(f, d, generator=g) * 0.02).to(dtype)
    b_in = (torch.randn(f, generator=g) * 0.05).to(dtype) if bias else None
    w_out = (torch.randn(d, f, generator=g) * 0.006).to(dtype)
    b_out = (torch.randn(d, generator=g) * 0.05).to(dtype) if bias else None
    return x, w_in, b_in, w_out, b_out


def _cuda(*ts):
    return [None if t is None else t.to(DEV) for t in ts]


def _kappa(x, w_in, b_in, density, dtype):
    z = omlp.linear(x, w_in, b_in).to(dtype)
    return og.round_kappa(max(0.0, og.kthvalue_threshold(z, density)), dtype)


GATES = [og.IDENTITY, og.GELU, og.ONE_SIDED, og.SYMMETRIC, og.RELU, og.GELU_MASKED, og.CORNER]
NAMES = {og.IDENTITY: "identity", og.GELU: "gelu", og.ONE_SIDED: "one_sided_threshold",
         og.SYMMETRIC: "symmetric_threshold", og.RELU: "relu", og.GELU_MASKED: "gelu_threshold",
         og.CORNER: "tile_corner_threshold"}


def _spec(op, kappa):
    from sparsity_spillover_b200.gates import from_mapping

    spec = {"operator": NAMES[op]}
    if op in (og.ONE_SIDED, og.SYMMETRIC, og.GELU_MASKED, og.CORNER):
        spec["kappa"] = kappa
    return from_mapping(spec)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("op", GATES)
@pytest.mark.parametrize("shape", [(1000, 256, 1024), (128, 128, 512), (77, 64, 320)])
def test_up_gate_matches_reference_gate_on_kernel_z(dtype, op, shape):
    from sparsity_spillover_b200 import ops

    t, d, f = shape
    x, w_in, b_in, _, _ = _inputs(t, d, f, dtype, seed=t + d + f + op)
    kappa = _kappa(x, w_in, b_in, 0.1, dtype)
    spec = _spec(op, kappa)
    xd, wd, bd = _cuda(x, w_in, b_in)
    z_k = torch.empty(t, f, dtype=dtype, device=DEV)
    h_k, bits_k = ops.up_gate(xd, wd, bd, spec, z_out=z_k, seq_len=t)
    torch.cuda.synchronize()
    z_k, h_k, bits_k = z_k.cpu(), h_k.cpu(), bits_k.cpu()

    # z within tolerance of the fp32 oracle (one rounding of an fp32-accumulated GEMM).
    z_ref = omlp.linear(x, w_in, b_in)
    assert omlp.max_rel_error(z_k, z_ref) <= TOL[dtype]

    # h is exactly the reference gate of the kernel's own z.
    k = spec.kappa_for(dtype)
    if op in (og.GELU, og.GELU_MASKED):
        ref = og.apply(z_k.float(), op, k).to(dtype)
        assert torch.equal(h_k != 0, ref != 0) or op == og.GELU
        assert (h_k.float() - ref.float()).abs().max() <= 2 * og.ulp(float(ref.float().abs().max()), dtype)
    else:
        ref = og.apply(z_k, op, k, seq_len=t)
        assert torch.equal(h_k, ref)

    # Tile bitmap bit-exact against the oracle's OR-reduction of h != 0.
    np.testing.assert_array_equal(bits_k.numpy().view(np.uint32), obit.tile_bits(h_k))

    # Decisions that differ from the fp32 oracle's sit within one ulp of kappa.
    if op in (og.ONE_SIDED, og.SYMMETRIC):
        mask_k = og.apply(z_k, op, k) != 0
        mask_r = og.apply(z_ref.to(dtype), op, k) != 0
        flips = mask_k != mask_r
        if flips.any():
            zf = z_k[flips].float().abs()
            assert float((zf - k).abs().max()) <= 2 * og.ulp(k, dtype)


@pytest.mark.parametrize("fill", [0xFFFFFFFF, "random"])
@pytest.mark.parametrize("t,d,f,density", [(1000, 128, 320, 0.002), (4096, 512, 2048, 0.0005), (300, 256, 1024, 0.1)])
def test_up_gate_rewrites_every_bitmap_bit(fill, t, d, f, density):
    """The up projection writes each bit of the bitmap set or clear (no clear launch
    before it): a buffer full of stale bits comes out equal to the oracle's bitmap, with
    dead 64-column groups, a partial last 16-row group, a partial last tile and unused
    bits above the last group of a word."""
    from sparsity_spillover_b200 import ops

    dtype = torch.float16
    x, w_in, b_in, _, _ = _inputs(t, d, f, dtype, seed=t + f)
    spec = _spec(og.ONE_SIDED, _kappa(x, w_in, b_in, density, dtype))
    xd, wd, bd = _cuda(x, w_in, b_in)
    n = ops.tile_bits_size(t, f)
    if fill == "random":
        g = torch.Generator().manual_seed(t)
        bits = torch.randint(-2**31, 2**31 - 1, (n,), generator=g, dtype=torch.int64).to(torch.int32).to(DEV)
    else:
        bits = torch.full((n,), -1, dtype=torch.int32, device=DEV)
    h = torch.empty(t, f, dtype=dtype, device=DEV)
    ops.up_gate(xd, wd, bd, spec, h=h, bits=bits)
    torch.cuda.synchronize()
    ref = obit.tile_bits(h.cpu())
    np.testing.assert_array_equal(bits.cpu().numpy().view(np.uint32), ref)
    live = obit.tile_mask(h.cpu())
    assert live.any()
    if density < 0.01:
        assert not live.all()  # dead groups too: their stale bits were cleared


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("density", [1.0, 0.25, 0.1, 0.02])
@pytest.mark.parametrize("skip", [True, "fine"])
def test_down_sparse_matches_fp32_oracle(dtype, density, skip):
    from sparsity_spillover_b200 import ops

    t, d, f = 1536, 512, 2048
    x, w_in, b_in, w_out, b_out = _inputs(t, d, f, dtype, seed=int(density * 100))
    kappa = _kappa(x, w_in, b_in, density, dtype)
    gate = {"operator": "one_sided_threshold", "kappa": kappa} if density < 1 else {"operator": "identity"}
    xd, wd, bd, wod, bod = _cuda(x, w_in, b_in, w_out, b_out)
    h, bits = ops.up_gate(xd, wd, bd, gate)
    stats = torch.zeros(2, dtype=torch.int64, device=DEV)
    y_skip = ops.down_sparse(h, bits, wod, bod, skip=skip, stats=stats)
    y_dense = ops.down_sparse(h, None, wod, bod, skip=False)
    torch.cuda.synchronize()
    h_c = h.cpu()
    y_ref = omlp.down_from_h(h_c, w_out, b_out)
    assert omlp.max_rel_error(y_skip.cpu(), y_ref) <= TOL[dtype]
    assert torch.equal(y_skip, y_dense)
    mask = obit.tile_mask(h_c)
    issued, skipped = obit.skip_counts(mask, f, n_tiles=(d + 255) // 256, m_tile=ops.down_tile_tokens(skip))
    assert stats.cpu().tolist() == [issued, skipped]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_residual_rounding_order(dtype):
    """y = round(round(h W^T + b) + r), the order of the reference's joint restatement."""
    from sparsity_spillover_b200 import ops

    t, d, f = 256, 256, 1024
    x, w_in, b_in, w_out, b_out = _inputs(t, d, f, dtype, seed=5)
    r = torch.randn(t, d).to(dtype)
    xd, wd, bd, wod, bod, rd = _cuda(x, w_in, b_in, w_out, b_out, r)
    h, bits = ops.up_gate(xd, wd, bd, {"operator": "relu"})
    y = ops.down_sparse(h, bits, wod, bod, rd).cpu()
    y0 = ops.down_sparse(h, bits, wod, bod).cpu()
    expect = (y0.float() + r.float()).to(dtype)
    assert torch.equal(y, expect)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_mlp_end_to_end_against_dtype_oracle(dtype):
    """Whole block vs the reference's PyTorch semantics in the same dtype (z rounded
    once, gate on the rounded z, fp32 accumulation), computed independently on the
    CPU: gate decisions differ only within one ulp of kappa, and y passes the
    rel-L2 / atol+rtol gate of measurement.py:11-23."""
    from sparsity_spillover_b200 import ops

    t, d, f = 2048, 512, 2048
    x, w_in, b_in, w_out, b_out = _inputs(t, d, f, dtype, seed=11)
    kappa = _kappa(x, w_in, b_in, 0.1, dtype)
    xd, wd, bd, wod, bod = _cuda(x, w_in, b_in, w_out, b_out)
    spec = {"operator": "one_sided_threshold", "kappa": kappa}
    z_k = torch.empty(t, f, dtype=dtype, device=DEV)
    ops.up_gate(xd, wd, bd, spec, z_out=z_k)
    y = ops.mlp_forward(xd, wd, bd, wod, bod, spec).cpu()
    z_ref, h_ref, y_ref = omlp.mlp_forward_dtype(x, w_in, b_in, w_out, b_out, og.ONE_SIDED, kappa, dtype)
    k = og.round_kappa(kappa, dtype)
    z_k = z_k.cpu()
    flips = (og.one_sided(z_k, k) != 0) != (h_ref != 0)
    assert float(flips.float().mean()) < 1e-3
    if flips.any():
        assert float((z_k[flips].float() - k).abs().max()) <= 2 * og.ulp(k, dtype)
    report = omlp.numerical_gate(y_ref, y)
    assert report["pass"], report


@pytest.mark.parametrize("skip", [True, "fine"])
def test_tile_structured_h_skips_dead_tiles(skip):
    """cfg2-style input: 64x64 tiles live with p=0.2; skip == dense, counters match the oracle."""
    from sparsity_spillover_b200 import ops, workloads

    t, d, f = 4096, 256, 1024
    h, frac = workloads.tile_structured_h(t, f, 0.2, seed=3, device=DEV, dtype=torch.bfloat16)
    g = torch.Generator().manual_seed(4)
    w_out = (torch.randn(d, f, generator=g) * 0.02).to(torch.bfloat16).to(DEV)
    b_out = (torch.randn(d, generator=g) * 0.02).to(torch.bfloat16).to(DEV)
    bits = ops.tile_bits_from_h(h)
    stats = torch.zeros(2, dtype=torch.int64, device=DEV)
    y = ops.down_sparse(h, bits, w_out, b_out, skip=skip, stats=stats)
    y_dense = ops.down_sparse(h, None, w_out, b_out, skip=False)
    torch.cuda.synchronize()
    h_c = h.cpu()
    np.testing.assert_array_equal(bits.cpu().numpy().view(np.uint32), obit.tile_bits(h_c))
    assert torch.equal(y, y_dense)
    assert omlp.max_rel_error(y.cpu(), omlp.down_from_h(h_c, w_out.cpu(), b_out.cpu())) <= TOL[torch.bfloat16]
    issued, skipped = obit.skip_counts(obit.tile_mask(h_c), f, n_tiles=1, m_tile=ops.down_tile_tokens(skip))
    assert stats.cpu().tolist() == [issued, skipped]
    assert skipped > 0


def test_all_zero_h_writes_bias_only():
    from sparsity_spillover_b200 import ops

    t, d, f = 300, 256, 512
    h = torch.zeros(t, f, dtype=torch.float16, device=DEV)
    w_out = torch.randn(d, f, dtype=torch.float16, device=DEV)
    b_out = torch.randn(d, dtype=torch.float16, device=DEV)
    bits = ops.tile_bits_from_h(h)
    stats = torch.zeros(2, dtype=torch.int64, device=DEV)
    y = ops.down_sparse(h, bits, w_out, b_out, stats=stats)
    assert int(bits.abs().sum()) == 0
    assert torch.equal(y, b_out.expand(t, d))
    assert int(stats[0]) == 0


def test_corner_gate_respects_sequences():
    """8x16 corner tiles restart at each sequence boundary (tile_gate.py:20-29)."""
    from sparsity_spillover_b200 import ops

    dtype = torch.bfloat16
    b, s, d, f = 3, 40, 128, 256
    x, w_in, b_in, _, _ = _inputs(b * s, d, f, dtype, seed=9)
    kappa = _kappa(x, w_in, b_in, 0.3, dtype)
    xd, wd, bd = _cuda(x, w_in, b_in)
    z = torch.empty(b * s, f, dtype=dtype, device=DEV)
    h, bits = ops.up_gate(xd, wd, bd, {"operator": "tile_corner_threshold", "kappa": kappa}, z_out=z, seq_len=s)
    z_c, h_c = z.cpu(), h.cpu()
    ref = og.corner(z_c.reshape(b, s, f), og.round_kappa(kappa, dtype)).reshape(b * s, f)
    assert torch.equal(h_c, ref)
    np.testing.assert_array_equal(bits.cpu().numpy().view(np.uint32), obit.tile_bits(h_c))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("b,s,d,f", [(7, 37, 128, 256), (5, 301, 256, 512), (3, 1000, 128, 1024)])
def test_corner_gate_partial_final_blocks(dtype, b, s, d, f):
    """Sequences whose length is not a multiple of 8 end with a shorter token block
    decided by its own first row (tile_gate.py:25-28): h equals the reference gate of
    the kernel's z with blocks restarting per sequence, the bitmap matches, and the
    down projection of that h matches the oracle."""
    from sparsity_spillover_b200 import ops

    t = b * s
    x, w_in, b_in, w_out, b_out = _inputs(t, d, f, dtype, seed=t + f)
    kappa = _kappa(x, w_in, b_in, 0.3, dtype)
    xd, wd, bd, wod, bod = _cuda(x, w_in, b_in, w_out, b_out)
    z = torch.empty(t, f, dtype=dtype, device=DEV)
    h, bits = ops.up_gate(xd, wd, bd, {"operator": "tile_corner_threshold", "kappa": kappa}, z_out=z, seq_len=s)
    y = ops.down_sparse(h, bits, wod, bod, skip="fine")
    torch.cuda.synchronize()
    z_c, h_c = z.cpu(), h.cpu()
    ref = og.corner(z_c.reshape(b, s, f), og.round_kappa(kappa, dtype)).reshape(t, f)
    assert torch.equal(h_c, ref)
    assert int((h_c != 0).sum()) > 0 and int((h_c == 0).sum()) > 0
    np.testing.assert_array_equal(bits.cpu().numpy().view(np.uint32), obit.tile_bits(h_c))
    y_ref = omlp.down_from_h(h_c, w_out, b_out)
    assert omlp.max_rel_error(y.cpu(), y_ref) <= TOL[dtype]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("skip", [True, "fine"])
def test_cfg3_shape_up_gate_and_down_sparse(dtype, skip):
    """The Pythia-410M layer shape (d=1024, F=4096) at 10 % element density on 2048
    tokens: h bit-exact against the gate of the kernel's z, the bitmap exact, z and y
    within tolerance of the fp32 oracle, and the skip counters equal to the oracle's."""
    from sparsity_spillover_b200 import ops

    t, d, f = 2048, 1024, 4096
    x, w_in, b_in, w_out, b_out = _inputs(t, d, f, dtype, seed=410)
    kappa = _kappa(x, w_in, b_in, 0.1, dtype)
    spec = _spec(og.ONE_SIDED, kappa)
    xd, wd, bd, wod, bod = _cuda(x, w_in, b_in, w_out, b_out)
    r = torch.randn(t, d, generator=torch.Generator().manual_seed(411)).to(dtype)
    z = torch.empty(t, f, dtype=dtype, device=DEV)
    h, bits = ops.up_gate(xd, wd, bd, spec, z_out=z)
    stats = torch.zeros(2, dtype=torch.int64, device=DEV)
    y = ops.down_sparse(h, bits, wod, bod, r.to(DEV), skip=skip, stats=stats)
    torch.cuda.synchronize()
    z_c, h_c = z.cpu(), h.cpu()
    assert omlp.max_rel_error(z_c, omlp.linear(x, w_in, b_in)) <= TOL[dtype]
    assert torch.equal(h_c, og.apply(z_c, og.ONE_SIDED, spec.kappa_for(dtype)))
    np.testing.assert_array_equal(bits.cpu().numpy().view(np.uint32), obit.tile_bits(h_c))
    y_ref = omlp.down_from_h(h_c, w_out, b_out, residual=r)
    assert omlp.max_rel_error(y.cpu(), y_ref) <= TOL[dtype]
    issued, skipped = obit.skip_counts(obit.tile_mask(h_c), f, n_tiles=d // 256, m_tile=ops.down_tile_tokens(skip))
    assert stats.cpu().tolist() == [issued, skipped]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("t,d,f,density", [(4096, 128, 512, 0.1), (1000, 128, 512, 0.01), (25600, 128, 512, 0.002)])
def test_small_shapes_take_narrow_tiles(dtype, t, d, f, density):
    """The 14M shape (d=128, F=512): the up projection runs 128 x 128 tiles on single CTAs
    when its pair tiles would not fill the GPU, and the down projection 128-column tiles
    on CTA pairs (T=25600: 100 pair tiles, the last round split into half-width items).  h, the bitmap, y and the skip counters are held to the same bars as
    the large shapes; the skipping y equals the dense y bit for bit."""
    from sparsity_spillover_b200 import ops

    x, w_in, b_in, w_out, b_out = _inputs(t, d, f, dtype, seed=14 + t)
    spec = _spec(og.ONE_SIDED, _kappa(x, w_in, b_in, density, dtype))
    xd, wd, bd, wod, bod = _cuda(x, w_in, b_in, w_out, b_out)
    r = torch.randn(t, d, generator=torch.Generator().manual_seed(15)).to(dtype)
    z = torch.empty(t, f, dtype=dtype, device=DEV)
    h, bits = ops.up_gate(xd, wd, bd, spec, z_out=z)
    stats = torch.zeros(2, dtype=torch.int64, device=DEV)
    y = ops.down_sparse(h, bits, wod, bod, r.to(DEV), skip=True, stats=stats)
    y_dense = ops.down_sparse(h, None, wod, bod, r.to(DEV), skip=False)
    torch.cuda.synchronize()
    z_c, h_c = z.cpu(), h.cpu()
    assert omlp.max_rel_error(z_c, omlp.linear(x, w_in, b_in)) <= TOL[dtype]
    assert torch.equal(h_c, og.apply(z_c, og.ONE_SIDED, spec.kappa_for(dtype)))
    np.testing.assert_array_equal(bits.cpu().numpy().view(np.uint32), obit.tile_bits(h_c))
    assert torch.equal(y, y_dense)
    assert omlp.max_rel_error(y.cpu(), omlp.down_from_h(h_c, w_out, b_out, residual=r, dtype=dtype)) <= TOL[dtype]
    issued, skipped = obit.skip_counts(obit.tile_mask(h_c), f, n_tiles=1, m_tile=ops.down_tile_tokens(True))
    assert stats.cpu().tolist() == [issued, skipped]


@pytest.mark.parametrize("skip", [True, "fine"])
def test_cfg2_full_size_tile_structured(skip):
    """cfg2 at its full size (T=65536, d=512, F=2048, bf16, 64x64 tiles live with p=0.1):
    the skipping down projection is bit-identical to its dense mode, its counters equal
    the oracle's tile accounting over all tokens, and two token ranges (the first and
    the last 2048 tokens) match the fp32 oracle."""
    from sparsity_spillover_b200 import ops, workloads

    t, d, f = 65536, 512, 2048
    h, _ = workloads.tile_structured_h(t, f, 0.1, seed=612, device=DEV, dtype=torch.bfloat16)
    g = torch.Generator().manual_seed(613)
    w_out = (torch.randn(d, f, generator=g) * 0.02).to(torch.bfloat16)
    b_out = (torch.randn(d, generator=g) * 0.02).to(torch.bfloat16)
    bits = ops.tile_bits_from_h(h)
    stats = torch.zeros(2, dtype=torch.int64, device=DEV)
    y = ops.down_sparse(h, bits, w_out.to(DEV), b_out.to(DEV), skip=skip, stats=stats)
    y_dense = ops.down_sparse(h, None, w_out.to(DEV), b_out.to(DEV), skip=False)
    torch.cuda.synchronize()
    assert torch.equal(y, y_dense)
    h_c = h.cpu()
    issued, skipped = obit.skip_counts(obit.tile_mask(h_c), f, n_tiles=d // 256, m_tile=ops.down_tile_tokens(skip))
    assert stats.cpu().tolist() == [issued, skipped]
    assert skipped > 0
    for rows in (slice(0, 2048), slice(t - 2048, t)):
        y_ref = omlp.down_from_h(h_c[rows], w_out, b_out, dtype=torch.bfloat16)
        assert omlp.max_rel_error(y.cpu()[rows], y_ref) <= TOL[torch.bfloat16]


def test_invalid_arguments_raise():
    from sparsity_spillover_b200 import ops
    from sparsity_spillover_b200._lib import SpmlpError

    x = torch.randn(64, 100, dtype=torch.float16, device=DEV)  # d not a multiple of 64
    w = torch.randn(128, 100, dtype=torch.float16, device=DEV)
    with pytest.raises(SpmlpError, match="multiple of 64"):
        ops.up_gate(x, w, None, {"operator": "relu"})
    with pytest.raises(ValueError):
        ops.up_gate(x.cpu(), w.cpu(), None, {"operator": "relu"})
    with pytest.raises(ValueError):
        ops.up_gate(x, w, None, {"operator": "one_sided_threshold", "kappa": -1.0})
    assert ops.device_status() == 0


def test_cfg1_full_size_properties():
    """The 70M shape at T=32768: bitmap and gate bit-exact on the full tensors,
    skip == dense, sampled rows of y against the fp32 oracle."""
    from sparsity_spillover_b200 import ops, workloads

    cfg = workloads.CONFIGS["cfg1"]
    layer = workloads.make_weights(cfg, DEV)[0]
    x = workloads.make_input(cfg, DEV)
    z = torch.empty(cfg.tokens, cfg.F, dtype=cfg.dtype, device=DEV)
    ops.up_gate(x, layer.w_in, layer.b_in, {"operator": "identity"}, z_out=z)
    kappa = workloads.quantile_threshold(z, 0.1)
    spec = {"operator": "one_sided_threshold", "kappa": kappa}
    h, bits = ops.up_gate(x, layer.w_in, layer.b_in, spec, z_out=z)
    y = ops.down_sparse(h, bits, layer.w_out, layer.b_out)
    y_dense = ops.down_sparse(h, None, layer.w_out, layer.b_out, skip=False)
    torch.cuda.synchronize()
    assert torch.equal(y, y_dense)
    z_c, h_c = z.cpu(), h.cpu()
    k = og.round_kappa(kappa, cfg.dtype)
    assert torch.equal(h_c, og.one_sided(z_c, k))
    np.testing.assert_array_equal(bits.cpu().numpy().view(np.uint32), obit.tile_bits(h_c))
    density = float((h_c != 0).float().mean())
    assert 0.09 < density < 0.11
    rows = torch.randperm(cfg.tokens, generator=torch.Generator().manual_seed(1))[:256]
    y_ref = omlp.down_from_h(h_c[rows], layer.w_out.cpu(), layer.b_out.cpu())
    assert omlp.max_rel_error(y.cpu()[rows], y_ref) <= TOL[cfg.dtype]
    z_ref = omlp.linear(x.cpu()[rows], layer.w_in.cpu(), layer.b_in.cpu())
    assert omlp.max_rel_error(z_c[rows], z_ref) <= TOL[cfg.dtype]
    assert ops.device_status() == 0


@pytest.mark.parametrize("graph", [False, True])
def test_pipelined_host_forward_matches_device_forward(graph):
    """Chunked host-to-host forward (copies overlapped with compute, optionally graph
    replayed) is bit-identical to the device forward: the MLP is token-local."""
    from sparsity_spillover_b200 import pipeline, workloads

    cfg = workloads.CONFIGS["cfg1"]
    ws = workloads.make_weights(cfg, DEV)[:3]
    layers = [pipeline.Layer(w.w_in, w.b_in, w.w_out, w.b_out, {"operator": "one_sided_threshold", "kappa": 0.5})
              for w in ws]
    stack = pipeline.MLPStack(layers)
    x = workloads.make_input(cfg, DEV, tokens=8192)
    y_dev = stack.forward(x).clone()
    x_host = x.cpu().pin_memory()
    y_host = torch.empty_like(x_host).pin_memory()
    for _ in range(2):  # first call runs eagerly (and captures), second replays
        y_host.zero_()
        stack.forward_host(x_host, y_host, chunks=4, graph=graph)
        torch.cuda.synchronize()
        assert torch.equal(y_host, y_dev.cpu())


def test_streamed_host_batches_match_device_forward():
    """Batch-pipelined host-to-host serving (double-buffered slots, graph replay):
    every batch's result equals the device forward of that batch."""
    from sparsity_spillover_b200 import pipeline, workloads

    cfg = workloads.CONFIGS["cfg1"]
    ws = workloads.make_weights(cfg, DEV)[:2]
    layers = [pipeline.Layer(w.w_in, w.b_in, w.w_out, w.b_out, {"operator": "one_sided_threshold", "kappa": 0.5})
              for w in ws]
    stack = pipeline.MLPStack(layers)
    xs = [workloads.make_input(cfg, DEV, tokens=4096, token_offset=i) for i in range(5)]
    expect = [stack.forward(x).clone().cpu() for x in xs]
    x_hosts = [x.cpu().pin_memory() for x in xs]
    y_hosts = [torch.empty_like(xh).pin_memory() for xh in x_hosts]
    for _ in range(2):
        stack.stream_host(x_hosts, y_hosts)
        torch.cuda.synchronize()
        for y, e in zip(y_hosts, expect):
            assert torch.equal(y, e)


@pytest.mark.parametrize("encoding", ["raw", "runs"])
def test_persisted_bitmap_drives_the_down_projection_identically(tmp_path, encoding):
    """A bitmap saved to disk and loaded back skips exactly the same K-tiles."""
    from sparsity_spillover_b200 import ops, workloads

    t, f, d = 8192, 2048, 512
    h, _ = workloads.tile_structured_h(t, f, 0.2, seed=31, device="cuda")
    w = (torch.randn(d, f, device="cuda") * 0.02).to(h.dtype)
    bits = ops.tile_bits_from_h(h)
    ops.save_mask(tmp_path / "mask.spmb", bits, t, f, encoding)
    loaded, t2, f2 = ops.load_mask(tmp_path / "mask.spmb", device="cuda")
    assert (t2, f2) == (t, f) and torch.equal(loaded, bits)
    st_a = torch.zeros(2, dtype=torch.int64, device="cuda")
    st_b = torch.zeros(2, dtype=torch.int64, device="cuda")
    y_a = ops.down_sparse(h, bits, w, None, stats=st_a)
    y_b = ops.down_sparse(h, loaded, w, None, stats=st_b)
    assert torch.equal(y_a, y_b) and torch.equal(st_a, st_b) and int(st_a[1]) > 0


def test_bounded_wait_times_out_reports_and_leaves_the_context_usable():
    """Failure detection without a fault: a wait that nothing completes gives up after
    ~2 s, the status word says which wait, and the GPU keeps working."""
    import time

    from sparsity_spillover_b200 import ops

    ops.clear_device_status()
    assert ops.device_status() == 0
    start = time.perf_counter()
    ops.selftest_wait()
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - start
    assert ops.device_status() == 5  # SPMLP_STATUS_TIMEOUT_PROBE
    assert 1.0 < elapsed < 30.0
    ops.clear_device_status()
    # The context still runs the kernels, with correct results.
    h = torch.zeros(64, 256, dtype=torch.float16, device="cuda")
    h[17, 70] = 1.0
    bits = ops.tile_bits_from_h(h)
    assert bits.cpu().tolist() == [0, 2, 0, 0]
    assert ops.device_status() == 0


@pytest.mark.parametrize("skip", [True, "fine"])
def test_last_round_split_tiles_match_the_oracle(skip):
    """At T=32768, d=512 the persistent grid's last round (coarse: 34 of 256 tiles on
    74 CTA pairs; fine: 68 of 512 on 148 CTAs) runs as half-width items: the final
    token blocks, both column halves, and the skip counts match the oracle."""
    from sparsity_spillover_b200 import ops, workloads

    t, d, f = 32768, 512, 2048
    h, _ = workloads.tile_structured_h(t, f, 0.2, seed=17, device=DEV, dtype=torch.bfloat16)
    g = torch.Generator().manual_seed(18)
    w_out = (torch.randn(d, f, generator=g) * 0.02).to(torch.bfloat16).to(DEV)
    b_out = (torch.randn(d, generator=g) * 0.02).to(torch.bfloat16).to(DEV)
    r = torch.randn(t, d, generator=g).to(torch.bfloat16).to(DEV)
    bits = ops.tile_bits_from_h(h)
    stats = torch.zeros(2, dtype=torch.int64, device=DEV)
    y = ops.down_sparse(h, bits, w_out, b_out, r, skip=skip, stats=stats)
    torch.cuda.synchronize()
    tail = slice(t - 4096, t)
    h_c = h.cpu()
    y_ref = omlp.down_from_h(h_c[tail], w_out.cpu(), b_out.cpu(), residual=r.cpu()[tail], dtype=torch.bfloat16)
    assert omlp.max_rel_error(y.cpu()[tail], y_ref) <= TOL[torch.bfloat16]
    issued, skipped = obit.skip_counts(obit.tile_mask(h_c), f, n_tiles=d // 256, m_tile=ops.down_tile_tokens(skip))
    assert stats.cpu().tolist() == [issued, skipped]


@pytest.mark.parametrize("sms", [2, 9, 100])
def test_sm_count_target_keeps_results_bit_identical(sms):
    """With the persistent GEMMs capped at a few SMs (as the pipelined d_ff split does while
    another stream's exchange runs), up_gate and every down mode give the same bits as
    uncapped; the cap is reset afterwards."""
    from sparsity_spillover_b200 import ops

    dtype, t, d, f = torch.float16, 2000, 512, 2048
    x, w_in, b_in, w_out, b_out = _inputs(t, d, f, dtype, seed=sms)
    spec = _spec(og.ONE_SIDED, _kappa(x, w_in, b_in, 0.1, dtype))
    xd, wd, bd, wod, bod = _cuda(x, w_in, b_in, w_out, b_out)

    def run():
        h, bits = ops.up_gate(xd, wd, bd, spec)
        ys = [ops.down_sparse(h, bits, wod, bod, xd, skip=s) for s in (False, True, "fine")]
        torch.cuda.synchronize()
        return [h, bits] + ys

    ref = run()
    try:
        ops.set_sm_count_target(sms)
        capped = run()
    finally:
        ops.set_sm_count_target(0)
    for a, b in zip(ref, capped):
        assert torch.equal(a, b)
    assert ops.device_status() == 0
