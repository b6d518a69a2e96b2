"""Multi-rank partition logic on CPU (gloo, world size 2): token shards and the
d_ff split with its reduce-scatter, with the kernel replaced by the oracle's
PyTorch restatement (the compute callable is injectable, like the reference
adapters' test backends)."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import gates as og
from oracle import mlp as omlp


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _oracle_partial(x, w_in, b_in, w_out, gate):
    z = omlp.linear(x, w_in, b_in).to(x.dtype)
    h = og.one_sided(z, gate)
    return omlp.linear(h, w_out, None).to(x.dtype)


def _worker(rank, world, port, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from sparsity_spillover_b200 import dist as sdist

        g = torch.Generator().manual_seed(11)
        t, d, f = 64, 64, 256
        x = torch.randn(t, d, generator=g).to(torch.bfloat16)
        w_in = (torch.randn(f, d, generator=g) * 0.1).to(torch.bfloat16)
        b_in = (torch.randn(f, generator=g) * 0.1).to(torch.bfloat16)
        w_out = (torch.randn(d, f, generator=g) * 0.05).to(torch.bfloat16)
        b_out = (torch.randn(d, generator=g) * 0.1).to(torch.bfloat16)
        r = torch.randn(t, d, generator=g).to(torch.bfloat16)
        kappa = og.round_kappa(0.2, torch.bfloat16)
        layer = sdist.DffSplitMLP.from_full(w_in, b_in, w_out, b_out, kappa, world, rank, compute=_oracle_partial)
        y = layer.forward(x, residual=r)
        lo, hi = sdist.token_shard(t, world, rank)
        _, _, y_full = omlp.mlp_forward_dtype(x, w_in, b_in, w_out, b_out, og.ONE_SIDED, kappa, torch.bfloat16)
        expect = (y_full.float() + r.float()).to(torch.bfloat16)[lo:hi]
        queue.put((rank, omlp.max_rel_error(y, expect), tuple(y.shape), (lo, hi)))
    finally:
        dist.destroy_process_group()


def test_dff_split_reduce_scatter_matches_single_process():
    world = 2
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = [queue.get(timeout=100) for _ in range(world)]
    for p in procs:
        p.join(timeout=30)
        assert p.exitcode == 0
    for rank, err, shape, (lo, hi) in sorted(results):
        assert shape == (32, 64)
        assert (lo, hi) == (rank * 32, rank * 32 + 32)
        assert err <= 1e-2  # bf16 partials are summed in a different order than on one GPU


def test_partition_helpers():
    from sparsity_spillover_b200 import dist as sdist

    assert [sdist.token_shard(10, 3, r) for r in range(3)] == [(0, 4), (4, 7), (7, 10)]
    assert sdist.dff_slice(4096, 8, 3) == (1536, 2048)
    with pytest.raises(ValueError):
        sdist.dff_slice(4096, 3, 0)


def test_pipelined_dff_split_rejects_uneven_slices():
    """Token slices must be equal: checked before any buffer or collective is set up."""
    from sparsity_spillover_b200 import dist as sdist

    for tokens, parts in ((1000, 3), (1024, 0)):
        with pytest.raises(ValueError):
            sdist.PipelinedDffSplit([], tokens, parts=parts)
