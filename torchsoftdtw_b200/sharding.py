"""Batch sharding across the GPUs of one node: one process per GPU (torchrun), pairs independent.

Soft-DTW pairs share nothing, so a global batch is cut into contiguous slices, one per rank, and each
rank runs the operator on its own slice with its inputs resident in its own HBM: the data path has no
collective at all. Two optional collectives exist for callers that want global results:

* :func:`all_reduce_loss` — the global loss sum (one scalar, ``all_reduce(SUM)``; NCCL over NVLink on
  CUDA, gloo on CPU); with ``async_op=True`` it returns at once with a handle, so the collective can run
  while the backward's kernels do (start it after the forward, wait on the handle after the backward);
* :func:`gather_costs` — every pair's cost on every rank (``all_gather`` of padded slices).
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def shard_bounds(B: int, world: int, rank: int) -> tuple[int, int]:
    """[begin, end) of rank's contiguous slice of a batch of B pairs; sizes differ by at most one."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad world/rank {world}/{rank}")
    base, extra = divmod(B, world)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)


def shard(t: torch.Tensor, world: int, rank: int) -> torch.Tensor:
    """Rank's slice of t along dim 0."""
    b, e = shard_bounds(t.shape[0], world, rank)
    return t[b:e]


class PendingSum:
    """An all-reduce in flight: :meth:`wait` makes the current stream wait for it and returns the sum."""

    def __init__(self, out: torch.Tensor, work):
        self._out = out
        self._work = work

    def wait(self) -> torch.Tensor:
        self._work.wait()
        return self._out


def all_reduce_loss(local_sum: torch.Tensor, group=None, async_op: bool = False):
    """Sum of every rank's local loss (in place on a clone; the input is left as it was).

    async_op=True returns a :class:`PendingSum` instead: the collective is enqueued behind the work already
    on the current stream (the forward that produced ``local_sum``) and runs beside whatever is enqueued
    next (the backward), until ``wait()`` joins it."""
    out = local_sum.detach().clone()
    work = dist.all_reduce(out, op=dist.ReduceOp.SUM, group=group, async_op=async_op)
    return PendingSum(out, work) if async_op else out


def gather_costs(local_costs: torch.Tensor, B: int, group=None) -> torch.Tensor:
    """Global (B,) costs on every rank, from each rank's contiguous slice."""
    world = dist.get_world_size(group)
    size = max(shard_bounds(B, world, r)[1] - shard_bounds(B, world, r)[0] for r in range(world))
    padded = torch.zeros(size, dtype=local_costs.dtype, device=local_costs.device)
    padded[: local_costs.shape[0]] = local_costs.detach()
    parts = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(parts, padded, group=group)
    out = [parts[r][: shard_bounds(B, world, r)[1] - shard_bounds(B, world, r)[0]] for r in range(world)]
    return torch.cat(out)
