"""Multi-GPU partitioning of the sparse gated MLP (one process per GPU, torch.distributed).

Two partitions:

* **Token sharding** — the MLP is token-local, so each rank runs the whole block
  on its own contiguous slice of tokens with replicated weights.  No collective
  is needed on the data path and the result is bit-identical to one GPU.

* **d_ff split** — rank r owns ``W_in[F_r, :]``, ``b_in[F_r]`` and ``W_out[:, F_r]``
  with ``F_r = [r F / w, (r + 1) F / w)``.  Every rank runs the fused up-projection +
  gate + bitmap and the tile-skipping down-projection on its slice for the same
  token block, producing a partial ``Y_r [T, d]``; a reduce-scatter over the token
  dimension sums the partials, and ``b_out`` (and the residual) are added once after
  the sum.  The bitmap stays rank-local: each slice's tiles are exactly the columns
  of the full bitmap for that slice.  ``DffSplitMLP`` / ``dff_split_forward`` do the
  reduce-scatter and the next layer's all-gather with NCCL; ``FusedDffSplit`` fuses
  them into the kernels: the down projection stores each partial tile straight into
  its owner's receive buffer over NVLink (peer memory from torch's symmetric memory)
  while later tiles still compute, and one reduction kernel per rank sums its block
  and writes the result into every rank's copy of the next layer's input.

The reference has no distributed code; this module is new.  The compute callable
is injectable (as the reference's adapters inject a PyTorch ``backend`` for tests,
runs/027-2026-09-06-pythia14m-kernel-sparsity-characterization/test_adapter.py:19-44), so
the partition and reduction logic is testable on CPU ranks with the gloo backend.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch
import torch.distributed as dist


def token_shard(tokens: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [start, end) token range of ``rank`` (sizes differ by at most one)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    base, extra = divmod(tokens, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def dff_slice(features: int, world: int, rank: int, granule: int = 64) -> tuple[int, int]:
    """[lo, hi) of rank's d_ff slice; slices are whole 64-feature bitmap columns."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    if features % (granule * world):
        raise ValueError(f"d_ff={features} must split into {world} slices of whole {granule}-feature tiles")
    per = features // world
    return rank * per, (rank + 1) * per


# compute(x, w_in, b_in, w_out, gate) -> partial y [T, d] in the activation dtype, without b_out.
PartialFn = Callable[[torch.Tensor, torch.Tensor, torch.Tensor | None, torch.Tensor, object], torch.Tensor]


def kernel_partial(x, w_in, b_in, w_out, gate):
    """Partial down-projection of one d_ff slice through libspmlp (up_gate + down_sparse)."""
    from . import ops

    h, bits = ops.up_gate(x, w_in, b_in, gate)
    return ops.down_sparse(h, bits, w_out, None)


@dataclass
class DffSplitMLP:
    """One rank's share of a d_ff-split gated MLP layer."""

    w_in: torch.Tensor   # [F/w, d]
    b_in: torch.Tensor | None
    w_out: torch.Tensor  # [d, F/w]
    b_out: torch.Tensor | None
    gate: object
    group: object = None
    compute: PartialFn = kernel_partial

    @classmethod
    def from_full(cls, w_in, b_in, w_out, b_out, gate, world: int, rank: int, group=None,
                  compute: PartialFn = kernel_partial) -> "DffSplitMLP":
        lo, hi = dff_slice(w_in.shape[0], world, rank)
        return cls(w_in[lo:hi].contiguous(), None if b_in is None else b_in[lo:hi].contiguous(),
                   w_out[:, lo:hi].contiguous(), b_out, gate, group, compute)

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
        """x [T, d] (the same on every rank) -> this rank's token block of y [T/w, d].

        y = round(round(sum_r Y_r + b_out) + residual), b_out added once after the sum."""
        world = dist.get_world_size(self.group)
        rank = dist.get_rank(self.group)
        t = x.shape[0]
        if t % world:
            raise ValueError(f"T={t} must divide evenly over {world} ranks for the reduce-scatter")
        partial = self.compute(x, self.w_in, self.b_in, self.w_out, self.gate)
        shard = reduce_scatter_tokens(partial, world, rank, self.group)
        lo, hi = rank * (t // world), (rank + 1) * (t // world)
        out = shard.float()
        if self.b_out is not None:
            out = out + self.b_out.float()
        y = out.to(x.dtype)
        if residual is not None:
            y = (y.float() + residual[lo:hi].float()).to(x.dtype)
        return y


def reduce_scatter_tokens(partial: torch.Tensor, world: int, rank: int, group=None) -> torch.Tensor:
    """Sum ``partial [T, d]`` over ranks and return this rank's [T/w, d] token block.

    NCCL runs a native reduce-scatter; backends without one (gloo, used by the CPU
    tests) all-reduce and keep their block.
    """
    t = partial.shape[0]
    per = t // world
    if dist.get_backend(group) == "nccl":
        out = torch.empty((per, partial.shape[1]), dtype=partial.dtype, device=partial.device)
        dist.reduce_scatter_tensor(out, partial.contiguous(), op=dist.ReduceOp.SUM, group=group)
        return out
    full = partial.clone()
    dist.all_reduce(full, op=dist.ReduceOp.SUM, group=group)
    return full[rank * per:(rank + 1) * per].contiguous()


def all_gather_tokens(shard: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """Concatenate every rank's [T/w, d] token block into the full [T, d] (rank order)."""
    out = torch.empty((shard.shape[0] * world, shard.shape[1]), dtype=shard.dtype, device=shard.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, shard.contiguous(), group=group)
    else:
        parts = [torch.empty_like(shard) for _ in range(world)]
        dist.all_gather(parts, shard.contiguous(), group=group)
        torch.cat(parts, out=out)
    return out


def dff_split_forward(layers: list[DffSplitMLP], x: torch.Tensor) -> torch.Tensor:
    """A stack of d_ff-split layers chained by the parallel residual, x_{l+1} = x_l + MLP_l(x_l).

    x [T, d] is the same on every rank; each layer reduce-scatters its partial
    down-projection over tokens and the next layer's input is all-gathered again.
    Returns this rank's [T/w, d] token block of the last layer's output."""
    if not layers:
        raise ValueError("need at least one layer")
    world = dist.get_world_size(layers[0].group)
    cur = x
    shard = None
    for i, layer in enumerate(layers):
        shard = layer.forward(cur, residual=cur)
        if i + 1 < len(layers):
            cur = all_gather_tokens(shard, world, layer.group)
    return shard


def multicast_available(device: torch.device) -> bool:
    """Whether torch symmetric memory on ``device`` can bind NVSwitch multicast objects."""
    from torch.distributed._symmetric_memory import DeviceType, _SymmetricMemory

    return device.type == "cuda" and bool(_SymmetricMemory.has_multicast_support(DeviceType.CUDA, device.index))


def _multicast_ok(handle) -> bool:
    """Whether a symmetric-memory rendezvous handle has an NVSwitch multicast mapping:
    the device supports multicast and the rendezvous produced a multicast address."""
    from torch.distributed._symmetric_memory import DeviceType, _SymmetricMemory

    device = handle.device
    if device.type != "cuda" or not _SymmetricMemory.has_multicast_support(DeviceType.CUDA, device.index):
        return False
    return int(handle.multicast_ptr or 0) != 0


class FusedDffSplit:
    """A stack of d_ff-split layers with the reduce-scatter and all-gather fused into
    the kernels (``spmlp_down_scatter`` / ``spmlp_reduce_broadcast``) over NVLink.

    Per layer: up_gate on the replicated input X (local); the scattering down
    projection writes rank r's partial of token block j into slot r of rank j's
    receive buffer; a one-element all-reduce orders it before every rank's
    reduction, which sums its block's slots in fp32, adds b_out and the residual
    (rounding like ``DffSplitMLP.forward``) and writes the block into every rank's X;
    a second barrier orders that before the next layer.  The barriers are
    ``spmlp_peer_barrier`` (epoch flags stored into peers' memory over NVLink, bounded
    waits); NCCL is used only once, to order the flags' initialisation.  X, the receive
    buffers and the flags are torch symmetric-memory tensors, so peers' addresses come
    from its rendezvous; tokens per rank must be a multiple of 256; one rank per GPU.

    ``multicast`` (NVLink SHARP): each rank's down projection writes its partial of
    all tokens into its own copy of a multicast-bound buffer; after the barrier,
    ``spmlp_reduce_broadcast_multicast`` reduces this rank's block inside the switch
    (multimem.ld_reduce) and writes the result to every rank's X (multimem.st).  Per
    rank and layer that moves the partial tokens once into the switch and the block
    once out of it, against (w-1)/w of the partials out and in again for the peer
    stores, so it pays from four ranks on.  None (default): multicast when the
    symmetric memory supports it and world >= 4.  Set False where a rank may die while
    the others run (a multicast-bound peer that disappears can fault the others).
    """

    MULTICAST_MIN_WORLD = 4

    def __init__(self, layers: list[DffSplitMLP], tokens: int, *, skip: bool | str = True,
                 multicast: bool | None = None):
        import torch.distributed._symmetric_memory as symm_mem

        from . import ops

        if not layers:
            raise ValueError("need at least one layer")
        self.layers = layers
        self.group = layers[0].group
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        if tokens % self.world or (tokens // self.world) % 256:
            raise ValueError(f"T={tokens} must split into {self.world} token blocks of a multiple of 256")
        w = layers[0].w_in
        self.device, self.dtype = w.device, w.dtype
        self.d, self.f = w.shape[1], w.shape[0]
        self.tokens, self.rows = tokens, tokens // self.world
        self.skip = skip
        group = self.group or dist.group.WORLD
        self.x = symm_mem.empty((tokens, self.d), dtype=self.dtype, device=self.device)
        hx = symm_mem.rendezvous(self.x, group)
        esize = self.x.element_size()
        block = self.rows * self.d * esize
        # A tensor may sit at an offset inside its symmetric buffer; peers' copies and the
        # multicast mapping put it at the same offset.
        off_x = self.x.data_ptr() - int(hx.buffer_ptrs[self.rank])
        supported = _multicast_ok(hx)
        if multicast is None:
            multicast = supported and self.world >= self.MULTICAST_MIN_WORLD
        if multicast and not supported:
            raise RuntimeError("symmetric memory on this system has no NVSwitch multicast support")
        self.multicast = bool(multicast)
        if self.multicast:
            # Partials of all tokens, one copy per rank, bound to a multicast object.
            self.part = symm_mem.empty((tokens, self.d), dtype=self.dtype, device=self.device)
            hr = symm_mem.rendezvous(self.part, group)
            if not _multicast_ok(hr):
                raise RuntimeError("the partial buffer got no multicast mapping")
            off_p = self.part.data_ptr() - int(hr.buffer_ptrs[self.rank])
            self.mc_part = int(hr.multicast_ptr) + off_p + self.rank * block  # my block, multicast addresses
            self.mc_x = int(hx.multicast_ptr) + off_x + self.rank * block
            self.slots = self.targets = []
        else:
            self.recv = symm_mem.empty((self.world, self.rows, self.d), dtype=self.dtype, device=self.device)
            hr = symm_mem.rendezvous(self.recv, group)
            off_r = self.recv.data_ptr() - int(hr.buffer_ptrs[self.rank])
            # My slot in each rank's receive buffer, and my token block in each rank's X.
            self.slots = [int(hr.buffer_ptrs[j]) + off_r + self.rank * block for j in range(self.world)]
            self.targets = [int(hx.buffer_ptrs[j]) + off_x + self.rank * block for j in range(self.world)]
        self.h = torch.empty((tokens, self.f), dtype=self.dtype, device=self.device)
        self.bits = torch.empty((ops.tile_bits_size(tokens, self.f),), dtype=torch.int32, device=self.device)
        self.flags = symm_mem.empty((self.world,), dtype=torch.int64, device=self.device)
        self.flags.zero_()
        hf = symm_mem.rendezvous(self.flags, group)
        off_f = self.flags.data_ptr() - int(hf.buffer_ptrs[self.rank])
        self.flag_slots = [int(hf.buffer_ptrs[j]) + off_f + self.rank * 8 for j in range(self.world)]
        self._handles = (hx, hr, hf)
        self.epoch = 0
        torch.cuda.synchronize(self.device)
        one = torch.zeros(1, dtype=torch.int32, device=self.device)
        dist.all_reduce(one, group=self.group)  # every rank's flags are zero before the first barrier
        torch.cuda.synchronize(self.device)

    def _barrier(self) -> None:
        from . import ops

        self.epoch += 1
        ops.peer_barrier(self.flag_slots, self.flags, self.epoch)

    def forward(self, x: torch.Tensor, *, check: bool = True) -> torch.Tensor:
        """x [T, d] (the same on every rank) -> this rank's [T/w, d] block of the last
        layer's output; the whole output is in ``self.x`` on every rank.

        A peer barrier that gives up (a peer did not signal within about 2 s: a slow,
        stuck or missing rank) lets the reduction run on partials that may be
        incomplete.  With ``check`` (default) the call waits for its kernels and raises
        ``PeerTimeoutError`` when the device status word reports such a failure; pass
        ``check=False`` inside timed loops and read ``ops.device_status`` afterwards."""
        self.begin(x)
        for i in range(len(self.layers)):
            self.layer_step(i)
        return self.finish(check)

    # The forward in steps, so that several instances (token slices) can interleave their
    # launches on their own streams (PipelinedDffSplit).  Every step launches on the
    # current stream.
    def begin(self, x: torch.Tensor) -> None:
        if tuple(x.shape) != (self.tokens, self.d):
            raise ValueError(f"x must be [{self.tokens}, {self.d}]")
        # The previous call ended with a barrier after every rank's last broadcast, so
        # overwriting X here races with no other rank.
        self.x.copy_(x)

    def layer_step(self, i: int) -> None:
        self.layer_gemms(i)
        self.layer_exchange(i)

    def layer_gemms(self, i: int) -> None:
        """Layer i's up_gate and (scattering) down projection: tensor-bound, local."""
        from . import ops

        layer = self.layers[i]
        ops.up_gate(self.x, layer.w_in, layer.b_in, layer.gate, h=self.h, bits=self.bits)
        if self.multicast:
            ops.down_sparse(self.h, self.bits, layer.w_out, None, None, skip=self.skip, y=self.part)
        else:
            ops.down_scatter(self.h, self.bits, layer.w_out, self.slots, skip=self.skip)

    def layer_exchange(self, i: int) -> None:
        """Layer i's barrier, reduction + broadcast and barrier: NVLink-bound, few SMs."""
        from . import ops

        layer = self.layers[i]
        mine = self.x[self.rank * self.rows:(self.rank + 1) * self.rows]
        self._barrier()
        if self.multicast:
            ops.reduce_broadcast_multicast(self.mc_part, self.mc_x, self.rows, self.d, layer.b_out, mine,
                                           self.dtype, self.device)
        else:
            ops.reduce_broadcast(self.recv, layer.b_out, mine, self.targets)
        self._barrier()

    def finish(self, check: bool = True) -> torch.Tensor:
        from . import ops

        mine = self.x[self.rank * self.rows:(self.rank + 1) * self.rows]
        if check:
            status = ops.device_status(self.device.index)
            if status != 0:
                raise PeerTimeoutError(self.rank, status)
        return mine


class PipelinedDffSplit:
    """The fused d_ff split over ``parts`` token slices, each a FusedDffSplit with its own
    buffers and barrier flags, launched layer by layer on its own CUDA stream, so that one
    slice's exchange (barrier, reduction + broadcast over NVLink: bandwidth-bound, few SMs)
    runs while the next slice's up and down projections (tensor-bound) run on the other SMs.

    The projections of all slices form one chain across the streams (slice p's projections
    of layer i start after slice p-1's, slice 0's of layer i+1 after the last slice's of
    layer i): run side by side they would only share the tensor cores and reach their
    exchanges together, with nothing left to overlap them.  The persistent GEMMs are
    capped at ``gemm_sms`` SMs (ops.set_sm_count_target; default: all but 40) during the
    forward, so that the exchange kernels always find SMs; 0 leaves them uncapped.  Slice
    p holds tokens [p T/parts, (p+1) T/parts); rank r's output is its block of every slice.

    Measured on 8 B200 (410M shape, 4 layers, 32768 tokens per rank, multicast exchange):
    the projections alone take 2.28 ms and the exchanges alone 5.54 ms; unsliced 8.07 ms,
    4 slices with the default cap 6.07 ms, so the projections hide behind the exchange.  On
    2 ranks (peer form) the exchange is short and slicing only adds barriers: there the
    unsliced FusedDffSplit is faster.
    A barrier waits only on the same slice's barrier of the other ranks, and every wait
    across ranks points to an earlier (layer, slice) step, so the launches cannot wait on
    one another in a cycle."""

    SM_RESERVE = 40  # SMs left to the exchange kernels while the projections run

    def __init__(self, layers: list[DffSplitMLP], tokens: int, *, parts: int = 4, gemm_sms: int | None = None,
                 skip: bool | str = True, multicast: bool | None = None):
        if parts < 1 or tokens % parts:
            raise ValueError(f"T={tokens} must split into {parts} equal token slices")
        self.parts = [FusedDffSplit(layers, tokens // parts, skip=skip, multicast=multicast) for _ in range(parts)]
        first = self.parts[0]
        self.device, self.tokens, self.d = first.device, tokens, first.d
        self.world, self.rank = first.world, first.rank
        props = torch.cuda.get_device_properties(self.device)
        self.gemm_sms = (max(1, props.multi_processor_count - self.SM_RESERVE) if gemm_sms is None
                         else int(gemm_sms))
        self.streams = [torch.cuda.Stream(self.device) for _ in range(parts)]
        self.multicast = first.multicast

    def forward(self, x: torch.Tensor, *, check: bool = True) -> list[torch.Tensor]:
        """x [T, d] (the same on every rank) -> this rank's output block of each slice
        (``parts`` tensors of [T / parts / world, d])."""
        from . import ops

        if tuple(x.shape) != (self.tokens, self.d):
            raise ValueError(f"x must be [{self.tokens}, {self.d}]")
        n = len(self.parts)
        rows = self.tokens // n
        main = torch.cuda.current_stream(self.device)
        start = torch.cuda.Event()
        start.record(main)
        ops.set_sm_count_target(self.gemm_sms, self.device.index)
        try:
            for p, (part, st) in enumerate(zip(self.parts, self.streams)):
                st.wait_event(start)
                with torch.cuda.stream(st):
                    part.begin(x[p * rows:(p + 1) * rows])
            gemms_done = None
            for i in range(len(self.parts[0].layers)):
                for part, st in zip(self.parts, self.streams):
                    with torch.cuda.stream(st):
                        if gemms_done is not None:
                            st.wait_event(gemms_done)
                        part.layer_gemms(i)
                        gemms_done = torch.cuda.Event()
                        gemms_done.record(st)
                        part.layer_exchange(i)
            for st in self.streams:
                ev = torch.cuda.Event()
                ev.record(st)
                main.wait_event(ev)
        finally:
            ops.set_sm_count_target(0, self.device.index)
        return [part.finish(check) for part in self.parts]


class PeerTimeoutError(RuntimeError):
    """A device-side wait of the fused d_ff split gave up (status word code ``code``,
    6 = a peer barrier whose peer did not signal in time); the layer outputs of that
    call are not valid.  The status word stays set until ``ops.clear_device_status``."""

    def __init__(self, rank: int, code: int):
        super().__init__(f"rank {rank}: fused d_ff split gave up waiting on the device (status {code}); "
                         "its output is not valid")
        self.rank = rank
        self.code = code
