"""Token sharding across GPUs (one process per GPU) and the error-statistics
reduction.

Encode, decode and the fused consumers treat token rows independently, so a
data-parallel job splits the rows of every activation evenly across ranks and
runs the whole path locally: no data crosses NVLink on the hot path.  The basis
and the outlier channel indices are replicated (computed once and broadcast, or
fitted identically on every rank).  The only collective is the reduction of
the reconstruction-error statistics that ``actcomp.error_stats`` produces per
rank: ``[sum (a-b)^2, sum b^2, max |a-b|, count(a != b)]`` -> sums of entries
0, 1, 3 and the maximum of entry 2 over all ranks.

Works with any ``torch.distributed`` backend: NCCL on GPUs (tensors on the
device), gloo on the CPU (tests run it with world size 2).
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist


def shard_rows(n_rows: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [start, stop) of rank ``rank`` when ``n_rows`` rows are split into
    ``world`` contiguous shards whose sizes differ by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    base, extra = divmod(n_rows, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard(x: torch.Tensor, world: Optional[int] = None, rank: Optional[int] = None, dim: int = -2) -> torch.Tensor:
    """This rank's contiguous slice of ``x`` along the token dimension ``dim``."""
    world = dist.get_world_size() if world is None else world
    rank = dist.get_rank() if rank is None else rank
    start, stop = shard_rows(x.shape[dim], world, rank)
    return x.narrow(dim, start, stop - start)


def reduce_error_stats(stats: torch.Tensor, group=None) -> torch.Tensor:
    """All-reduce the 4-entry statistics of ``actcomp.error_stats`` in place:
    entries 0, 1, 3 summed, entry 2 (max |a - b|) maximised.  Returns ``stats``."""
    if stats.numel() != 4:
        raise ValueError("expected the 4 entries of actcomp.error_stats")
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return stats
    mx = stats[2:3].clone()
    stats[2] = 0
    dist.all_reduce(stats, op=dist.ReduceOp.SUM, group=group)
    dist.all_reduce(mx, op=dist.ReduceOp.MAX, group=group)
    stats[2] = mx[0]
    return stats


def relative_error(stats: torch.Tensor) -> float:
    """||a - b||_F / ||b||_F from (reduced) statistics."""
    sse, ssb = float(stats[0]), float(stats[1])
    return (sse / ssb) ** 0.5 if ssb > 0 else 0.0
