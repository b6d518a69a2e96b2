"""Multi-GPU partitioning of the sparse gated MLP (one process per GPU, torch.distributed).

Two partitions:

* **Token sharding** — the MLP is token-local, so each rank runs the whole block
  on its own contiguous slice of tokens with replicated weights.  No collective
  is needed on the data path and the result is bit-identical to one GPU.

* **d_ff split** — rank r owns ``W_in[F_r, :]``, ``b_in[F_r]`` and ``W_out[:, F_r]``
  with ``F_r = [r F / w, (r + 1) F / w)``.  Every rank runs the fused up-projection +
  gate + bitmap and the tile-skipping down-projection on its slice for the same
  token block, producing a partial ``Y_r [T, d]``; a reduce-scatter over the token
  dimension (NCCL over NVLink on B200) sums the partials, and ``b_out`` (and the
  residual) are added once after the sum.  The bitmap stays rank-local: each slice's
  tiles are exactly the columns of the full bitmap for that slice.

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
