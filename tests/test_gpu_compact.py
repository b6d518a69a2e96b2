"""GPU parity of the compact down modes (SPMLP_DOWN_COMPACT / _FINE): live 16-feature
granules gathered into the pipeline stages.

* the 16x16 bitmap of spmlp_tile_bits16_from_h is bit-exact against the oracle's
  OR-reduction of h != 0 over 16x16 tiles;
* y is bit-identical to the dense mode (skipped granules contribute exact zeros) and
  within the north-star tolerance of the fp32 oracle;
* the issued / skipped K16 counters equal the oracle's accounting at 16-feature
  granules over each mode's token tile (runs/042-2026-09-20-pythia70m-sparse-scale/tile_oracle.py:4-20
  restated for these tiles).
Inputs carry the structure of the reference's corner-tile gate (8-token x 16-feature
tiles kept whole), where 16-feature granules skip far more than 64-feature K-blocks.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import bitmap as obit
from oracle import mlp as omlp

pytestmark = pytest.mark.gpu

TOL = {torch.float16: 2e-3, torch.bfloat16: 1e-2}
DEV = "cuda"


def _weights(d, f, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(d, f, generator=g) * 0.02).to(dtype)
    b = (torch.randn(d, generator=g) * 0.02).to(dtype)
    return w, b, g


@pytest.mark.parametrize("t,f", [(1000, 512), (77, 320), (4096, 2048)])
def test_tile_bits16_match_the_oracle(t, f):
    from sparsity_spillover_b200 import ops, workloads

    h, _ = workloads.corner_tile_h(t, f, 0.1, seed=t + f, device=DEV)
    h[3, 17] = -0.0  # -0.0 counts as zero
    bits = ops.tile_bits16_from_h(h)
    np.testing.assert_array_equal(bits.cpu().numpy().view(np.uint32), obit.tile_bits(h.cpu(), 16, 16))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("skip", ["compact", "compact_fine"])
@pytest.mark.parametrize("t,d,f,p", [(1000, 512, 2048, 0.05), (4096, 256, 1024, 0.2), (300, 512, 2048, 0.01)])
def test_compact_down_is_exact_and_counts_live_granules(dtype, skip, t, d, f, p):
    from sparsity_spillover_b200 import ops, workloads

    h, _ = workloads.corner_tile_h(t, f, p, seed=7 * t + f, device=DEV, dtype=dtype)
    w_out, b_out, g = _weights(d, f, dtype, seed=t + d)
    r = torch.randn(t, d, generator=g).to(dtype)
    wd, bd, rd = w_out.to(DEV), b_out.to(DEV), r.to(DEV)
    bits16 = ops.tile_bits16_from_h(h)
    stats = torch.zeros(2, dtype=torch.int64, device=DEV)
    y = ops.down_sparse(h, bits16, wd, bd, rd, skip=skip, stats=stats)
    y_dense = ops.down_sparse(h, None, wd, bd, rd, skip=False)
    torch.cuda.synchronize()
    assert torch.equal(y, y_dense)
    h_c = h.cpu()
    y_ref = omlp.down_from_h(h_c, w_out, b_out, residual=r, dtype=dtype)
    assert omlp.max_rel_error(y.cpu(), y_ref) <= TOL[dtype]
    issued, skipped = obit.skip_counts(obit.tile_mask(h_c, 16, 16), f, n_tiles=d // 256 if d >= 256 else 1,
                                       m_tile=ops.down_tile_tokens(skip), granule=16)
    assert stats.cpu().tolist() == [issued, skipped]
    assert skipped > 0


@pytest.mark.parametrize("skip", ["compact", "compact_fine"])
def test_compact_down_full_size_tail(skip):
    """T=32768 (the persistent grid's last round split into half-width items): the tail
    tokens match the oracle and the counters match over all tokens."""
    from sparsity_spillover_b200 import ops, workloads

    dtype, t, d, f = torch.bfloat16, 32768, 512, 2048
    h, _ = workloads.corner_tile_h(t, f, 0.02, seed=31, device=DEV, dtype=dtype)
    w_out, b_out, _ = _weights(d, f, dtype, seed=32)
    bits16 = ops.tile_bits16_from_h(h)
    stats = torch.zeros(2, dtype=torch.int64, device=DEV)
    y = ops.down_sparse(h, bits16, w_out.to(DEV), b_out.to(DEV), skip=skip, stats=stats)
    torch.cuda.synchronize()
    h_c = h.cpu()
    tail = slice(t - 4096, t)
    y_ref = omlp.down_from_h(h_c[tail], w_out, b_out, dtype=dtype)
    assert omlp.max_rel_error(y.cpu()[tail], y_ref) <= TOL[dtype]
    issued, skipped = obit.skip_counts(obit.tile_mask(h_c, 16, 16), f, n_tiles=d // 256,
                                       m_tile=ops.down_tile_tokens(skip), granule=16)
    assert stats.cpu().tolist() == [issued, skipped]


def test_compact_needs_its_bitmap():
    from sparsity_spillover_b200 import ops

    h = torch.zeros(64, 2048, dtype=torch.float16, device=DEV)
    w = torch.zeros(256, 2048, dtype=torch.float16, device=DEV)
    with pytest.raises(ValueError):
        ops.down_sparse(h, ops.tile_bits_from_h(h), w, None, skip="compact")  # a 16x64 bitmap has the wrong size
