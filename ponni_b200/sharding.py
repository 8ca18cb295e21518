"""Column sharding of a batch across the ranks of one node (weak scaling).

Samples (batch columns) are independent, so rank r of `world` owns the
global columns [r * per_rank, (r + 1) * per_rank) and no data crosses ranks;
the only collective is the reduction of each rank's timing to the job's
(the slowest rank's) time, outside the timed region.
"""
from __future__ import annotations


def shard_range(rank: int, world: int, per_rank: int) -> tuple[int, int]:
    """First global column and column count of `rank`'s shard."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if per_rank <= 0:
        raise ValueError("each rank needs a nonzero number of columns")
    return rank * per_rank, per_rank


def job_time(seconds: float, world: int, device=None) -> float:
    """The job's time: the maximum of every rank's `seconds` (all ranks call)."""
    if world <= 1:
        return float(seconds)
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(seconds)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
