"""GPU parity of the vocabulary head (embed_out) against the CPU oracle.

* dense: logits within the north-star tolerance of the fp32 oracle at the real
  vocabulary size V = 50304;
* K gate (the reference's head, runs/068-…/inference/head.cu): the prepared input
  and its 16x16 support bits are bit-exact against the oracle's fp32 corner
  certificates; logits match the oracle on the gated input; issued / skipped
  K16 steps match the oracle's accounting;
* N gate (vocabulary tiles): listed 128-column tiles are computed, every other
  logit is left untouched, and head_fill masks them.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import bitmap as obit
from oracle import head as ohead
from oracle import mlp as omlp

pytestmark = pytest.mark.gpu

TOL = {torch.float16: 2e-3, torch.bfloat16: 1e-2}
V = 50304


def _weights(d, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(V, d, generator=g) * 0.02).to(dtype)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("t,d", [(512, 128), (300, 512)])
def test_dense_head_matches_fp32_oracle(dtype, t, d):
    from sparsity_spillover_b200 import ops

    g = torch.Generator().manual_seed(t + d)
    x = torch.randn(t, d, generator=g).to(dtype)
    w = _weights(d, dtype, seed=d)
    logits = ops.head_sparse(x.cuda(), w.cuda()).cpu()
    ref = ohead.logits(x, w)
    assert omlp.max_rel_error(logits, ref) <= TOL[dtype]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("t,d", [(640, 128), (300, 512), (100, 1024)])
def test_k_gated_head_matches_reference_certificates(dtype, t, d):
    """The K-gated head (two vocabulary tiles per single-CTA item at every d): several
    32-granule chunks of support bits (d >= 512) and a partial last token block."""
    from sparsity_spillover_b200 import ops

    kappa = 0.1
    g = torch.Generator().manual_seed(68 + d)
    x = torch.randn(t, d, generator=g)
    corners = x[::16, ::16]
    corners[torch.rand(corners.shape, generator=g) < 0.8] = -1.0  # most tiles dead: whole K16 steps skip
    x[::16, ::16] = corners
    x[16, 32] = float(torch.nextafter(torch.tensor(kappa), torch.tensor(1.0)))  # survives in fp32 only
    w = _weights(d, dtype, seed=5)
    x_out, support = ops.head_prepare(x.cuda(), kappa, dtype)
    stats = torch.zeros(2, dtype=torch.int64, device="cuda")
    logits = ops.head_sparse(x_out, w.cuda(), support=support, stats=stats).cpu()
    ref_x, ref_bits = ohead.prepare(x, kappa, dtype)
    assert torch.equal(x_out.cpu(), ref_x)
    np.testing.assert_array_equal(support.cpu().numpy().view(np.uint32), ref_bits)
    assert omlp.max_rel_error(logits, ohead.logits(ref_x, w)) <= TOL[dtype]
    mask = ohead.support_mask(x, kappa)
    issued, skipped = obit.skip_counts(mask, d, n_tiles=V // 128, granule=16)
    assert stats.cpu().tolist() == [issued, skipped]
    assert skipped > 0 and issued > 0


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_n_gated_head_writes_only_active_vocabulary_tiles(dtype):
    from sparsity_spillover_b200 import ops, workloads

    t, d = 384, 512
    g = torch.Generator().manual_seed(9)
    x = torch.randn(t, d, generator=g).to(dtype)
    w = _weights(d, dtype, seed=3)
    tiles = workloads.zipf_active_tiles(V // 128, 0.1, seed=4)
    sentinel = torch.full((t, V), 7.0, dtype=dtype, device="cuda")
    logits = ops.head_sparse(x.cuda(), w.cuda(), active_tiles=torch.from_numpy(tiles).cuda(), logits=sentinel)
    out = logits.cpu()
    cols = np.concatenate([np.arange(k * 128, (k + 1) * 128) for k in tiles])
    ref = ohead.logits(x, w[cols])
    assert omlp.max_rel_error(out[:, cols], ref) <= TOL[dtype]
    inactive = np.setdiff1d(np.arange(V), cols)
    assert bool((out[:, inactive] == 7.0).all())
    dead = np.setdiff1d(np.arange(V // 128), tiles).astype(np.int32)
    ops.head_fill(logits, torch.from_numpy(dead).cuda(), float("-inf"))
    out2 = logits.cpu()
    assert bool(torch.isneginf(out2[:, inactive]).all())
    assert torch.equal(out2[:, cols], out[:, cols])


def test_sparse_head_module_masks_inactive_tiles():
    from sparsity_spillover_b200 import SparseHead, workloads

    d = 128
    lin = torch.nn.Linear(d, V, bias=False).half().cuda()
    tiles = workloads.zipf_active_tiles(V // 128, 0.05, seed=1)
    head = SparseHead(lin, active_tiles=tiles, masked_value=float("-inf"))
    x = torch.randn(2, 64, d, dtype=torch.float16, device="cuda")
    with torch.inference_mode():
        out = head(x)
    assert out.shape == (2, 64, V)
    cols = np.concatenate([np.arange(k * 128, (k + 1) * 128) for k in tiles])
    ref = ohead.logits(x.reshape(-1, d).cpu(), lin.weight.detach().cpu()[cols])
    assert omlp.max_rel_error(out.reshape(-1, V)[:, cols].cpu(), ref) <= TOL[torch.float16]
    assert bool(torch.isneginf(out.reshape(-1, V)[:, np.setdiff1d(np.arange(V), cols)]).all())


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("t,d", [(200, 128), (320, 512), (768, 512), (100, 1024)])
@pytest.mark.parametrize("n_active", [1, 2, 3, 8])
def test_n_gated_head_pairs_of_vocabulary_tiles(dtype, t, d, n_active):
    """The dense and N-gated head run two listed vocabulary tiles per work item, on a CTA
    pair from d = 512 and on one CTA below (d = 128 here): odd lists (a lone last tile),
    unsorted and non-adjacent tiles, token counts that leave a partial 256-token block;
    stats count per 128-token x 128-column tile in both forms."""
    from sparsity_spillover_b200 import ops

    g = torch.Generator().manual_seed(7 * t + n_active)
    x = torch.randn(t, d, generator=g).to(dtype)
    w = _weights(d, dtype, seed=11)
    tiles = torch.randperm(V // 128, generator=g)[:n_active].to(torch.int32)  # unsorted, scattered
    sentinel = torch.full((t, V), 5.0, dtype=dtype, device="cuda")
    stats = torch.zeros(2, dtype=torch.int64, device="cuda")
    logits = ops.head_sparse(x.cuda(), w.cuda(), active_tiles=tiles.cuda(), logits=sentinel, stats=stats)
    out = logits.cpu()
    cols = np.concatenate([np.arange(k * 128, (k + 1) * 128) for k in tiles.tolist()])
    ref = ohead.logits(x, w[cols])
    assert omlp.max_rel_error(out[:, cols], ref) <= TOL[dtype]
    assert bool((out[:, np.setdiff1d(np.arange(V), cols)] == 5.0).all())
    m_tiles = -(-t // 128)
    assert stats.cpu().tolist() == [n_active * m_tiles * (d // 16), 0]
