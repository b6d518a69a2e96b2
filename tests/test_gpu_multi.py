"""Two-GPU checks (skipped with fewer GPUs): the d_ff split with an NCCL
reduce-scatter over NVLink, and the fused d_ff split (partials stored into the
owner's buffer by the down projection, reduction + broadcast kernel), match one
GPU within tolerance on every rank's block and on the broadcast full output;
token shards are bit-identical to the single-GPU forward of the same tokens."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, queue):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from oracle import mlp as omlp
        from sparsity_spillover_b200 import dist as sdist
        from sparsity_spillover_b200 import ops, workloads

        cfg = workloads.CONFIGS["cfg3"]
        t = 4096
        full = workloads.make_weights(cfg, dev)[:2]
        gate = {"operator": "one_sided_threshold", "kappa": 0.5}
        x = workloads.make_input(cfg, dev, tokens=t)
        layers = [sdist.DffSplitMLP.from_full(L.w_in, L.b_in, L.w_out, L.b_out, gate, world, rank) for L in full]
        y_shard = sdist.dff_split_forward(layers, x)
        # single-GPU reference of the same two layers on this rank's device
        ref = x
        for L in full:
            ref = ops.mlp_forward(ref, L.w_in, L.b_in, L.w_out, L.b_out, gate, residual=ref)
        lo, hi = rank * t // world, (rank + 1) * t // world
        err = omlp.max_rel_error(y_shard.float().cpu(), ref[lo:hi].float().cpu())
        # One layer against the one-GPU layer: the north-star bar (fp16 2e-3).  Over the
        # two-layer chain the forms' different rounding of partial sums can flip gate
        # decisions at kappa in layer 2, hence the looser chained bound below.
        ref1 = ops.mlp_forward(x, full[0].w_in, full[0].b_in, full[0].w_out, full[0].b_out, gate, residual=x)
        err1 = omlp.max_rel_error(sdist.dff_split_forward(layers[:1], x).float().cpu(), ref1[lo:hi].float().cpu())
        fused1 = sdist.FusedDffSplit(layers[:1], t, multicast=False)
        err1_fused = omlp.max_rel_error(fused1.forward(x).float().cpu(), ref1[lo:hi].float().cpu())
        err1 = max(err1, err1_fused)
        # token sharding: this rank's shard through the unsplit layer equals the full pass's rows
        tok = ops.mlp_forward(x[lo:hi].contiguous(), full[0].w_in, full[0].b_in, full[0].w_out, full[0].b_out, gate)
        whole = ops.mlp_forward(x, full[0].w_in, full[0].b_in, full[0].w_out, full[0].b_out, gate)
        same = bool(torch.equal(tok, whole[lo:hi]))
        # the fused d_ff split: P2P scatter from the down projection, reduction + broadcast kernel
        fused = sdist.FusedDffSplit(layers, t, multicast=False)  # peer stores (the failure test below)
        y_fused = fused.forward(x)
        err_fused = omlp.max_rel_error(y_fused.float().cpu(), ref[lo:hi].float().cpu())
        full_x = fused.x.clone()
        # The same layers as four token slices on four streams (PipelinedDffSplit): each
        # rank's block of each slice equals the unsliced fused split's rows (peer form: the
        # reduction sums in rank order in both).
        pipe = sdist.PipelinedDffSplit(layers, t, parts=4, multicast=False)
        blocks = pipe.forward(x)
        span, sub = t // 4, t // 4 // world
        rows_of = [slice(p * span + rank * sub, p * span + (rank + 1) * sub) for p in range(4)]
        pipe_same = all(bool(torch.equal(b, full_x[sl])) for b, sl in zip(blocks, rows_of))
        pipe_err = max(omlp.max_rel_error(b.float().cpu(), ref[sl].float().cpu()) for b, sl in zip(blocks, rows_of))
        y_again = fused.forward(x).clone()  # a second call reuses the buffers and gives the same result
        same_again = bool(torch.equal(y_again, y_fused)) and bool(torch.equal(fused.x, full_x))
        rows_ok = omlp.max_rel_error(full_x.float().cpu(), ref.float().cpu())  # every block reached every rank
        torch.cuda.synchronize(dev)
        status = ops.device_status(rank)
        # Failure detection without a fault: rank 0 waits for an epoch that rank 1 never
        # signals; the bounded wait gives up, the status word says so, the GPU keeps working.
        timeout_status, usable, raised = 6, True, True
        if rank == 0:
            ops.clear_device_status(rank)
            ops.peer_barrier(fused.flag_slots, fused.flags, fused.epoch + 1000)
            torch.cuda.synchronize(dev)
            timeout_status = ops.device_status(rank)
            ops.clear_device_status(rank)
            probe = torch.zeros(64, 128, dtype=torch.float16, device=dev)
            probe[5, 70] = 1.0
            usable = ops.tile_bits_from_h(probe).cpu().tolist() == [2, 0, 0, 0]
            # A whole forward while rank 1 stays out: its barriers give up, and forward
            # reports it instead of returning the incomplete result.
            try:
                fused.forward(x)
                raised = False
            except sdist.PeerTimeoutError as exc:
                raised = exc.code == 6
            ops.clear_device_status(rank)
        queue.put((rank, err, same, status, err_fused, same_again, rows_ok, timeout_status, usable and raised, err1,
                   pipe_err, pipe_same))
    finally:
        dist.barrier(device_ids=[rank])
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_dff_split_over_nccl_and_token_shards():
    world = 2
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = [queue.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for (rank, err, same, status, err_fused, same_again, rows_ok, timeout_status, usable, err1,
         pipe_err, pipe_same) in results:
        assert err1 <= 2e-3, (rank, err1)  # one layer, NCCL and fused forms
        assert err <= 2e-2, (rank, err)  # fp16 partials summed by NCCL, then bias and residual rounding
        assert same
        assert status == 0
        assert err_fused <= 2e-2, (rank, err_fused)  # fp16 partials summed in fp32
        assert same_again
        assert rows_ok <= 2e-2, (rank, rows_ok)
        assert timeout_status == 6 and usable  # SPMLP_STATUS_TIMEOUT_PEER
        assert pipe_err <= 2e-2, (rank, pipe_err)
        assert pipe_same  # per token, the sliced run computes exactly what the unsliced one does


def _multicast_worker(rank, world, port, queue):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        import torch.distributed._symmetric_memory as symm_mem

        from oracle import mlp as omlp
        from sparsity_spillover_b200 import dist as sdist
        from sparsity_spillover_b200 import ops, workloads

        probe = symm_mem.empty((256,), dtype=torch.float16, device=dev)
        supported = sdist._multicast_ok(symm_mem.rendezvous(probe, dist.group.WORLD))
        result = {"rank": rank, "supported": supported}
        if supported:
            cfg = workloads.CONFIGS["cfg3"]
            t = 4096
            full = workloads.make_weights(cfg, dev)[:2]
            gate = {"operator": "one_sided_threshold", "kappa": 0.5}
            x = workloads.make_input(cfg, dev, tokens=t)
            layers = [sdist.DffSplitMLP.from_full(L.w_in, L.b_in, L.w_out, L.b_out, gate, world, rank) for L in full]
            ref = x
            for L in full:
                ref = ops.mlp_forward(ref, L.w_in, L.b_in, L.w_out, L.b_out, gate, residual=ref)
            lo, hi = rank * t // world, (rank + 1) * t // world
            mc = sdist.FusedDffSplit(layers, t, multicast=True)
            y = mc.forward(x).clone()
            full_x = mc.x.clone()
            y2 = mc.forward(x).clone()
            peer = sdist.FusedDffSplit(layers, t, multicast=False)
            y_peer = peer.forward(x).clone()
            # one layer against the one-GPU layer
            ref1 = ops.mlp_forward(x, full[0].w_in, full[0].b_in, full[0].w_out, full[0].b_out, gate, residual=x)
            mc1 = sdist.FusedDffSplit(layers[:1], t, multicast=True)
            err1 = omlp.max_rel_error(mc1.forward(x).float().cpu(), ref1[lo:hi].float().cpu())
            # the same layer as four token slices on four streams, projections capped
            pipe1 = sdist.PipelinedDffSplit(layers[:1], t, parts=4, multicast=True)
            span, sub = t // 4, t // 4 // world
            rows_of = [slice(p * span + rank * sub, p * span + (rank + 1) * sub) for p in range(4)]
            err1_pipe = max(omlp.max_rel_error(b.float().cpu(), ref1[sl].float().cpu())
                            for b, sl in zip(pipe1.forward(x), rows_of))
            torch.cuda.synchronize(dev)
            result.update(multicast=mc.multicast and pipe1.multicast, err1=max(err1, err1_pipe),
                          err=omlp.max_rel_error(y.float().cpu(), ref[lo:hi].float().cpu()),
                          rows_ok=omlp.max_rel_error(full_x.float().cpu(), ref.float().cpu()),
                          same_again=bool(torch.equal(y, y2)),
                          vs_peer=omlp.max_rel_error(y.float().cpu(), y_peer.float().cpu()),
                          status=ops.device_status(rank))
        queue.put(result)
    finally:
        dist.barrier(device_ids=[rank])
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_fused_dff_split_through_nvswitch_multicast():
    """The d_ff split's reduction + broadcast through NVLink SHARP (multimem.ld_reduce,
    multimem.st) matches one GPU and the peer-store form within tolerance, gives the
    same result on a second call, and leaves every block on every rank.  No rank fails
    here: failure detection runs on the peer-store form only."""
    world = 2
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_multicast_worker, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = [queue.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    if not all(r["supported"] for r in results):
        pytest.skip("no NVSwitch multicast support for symmetric memory on this system")
    for r in results:
        assert r["multicast"] and r["status"] == 0
        assert r["err1"] <= 2e-3, r  # one layer
        assert r["err"] <= 2e-2, r  # fp16 partials reduced in fp32 in the switch, rounded, then bias / residual
        assert r["rows_ok"] <= 2e-2, r
        assert r["same_again"], r
        assert r["vs_peer"] <= 2e-2, r
