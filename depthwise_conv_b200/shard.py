"""Batch sharding across the GPUs of one node (one process per GPU, no collectives).

Images are independent, so rank r of N processes the contiguous batch slice
``shard_range(B, N, r)``; a batch smaller than N leaves the last ranks idle.
Throughput is the images of all ranks over the slowest rank's time, which
``max_over_ranks`` computes with one all-reduce (MAX) outside the timed region.
"""
from __future__ import annotations


def shard_range(batch: int, world: int, rank: int) -> tuple[int, int]:
    """[start, end) of rank's slice: sizes differ by at most one, lower ranks larger."""
    if world < 1 or not 0 <= rank < world or batch < 0:
        raise ValueError(f"bad shard request batch={batch} world={world} rank={rank}")
    base, extra = divmod(batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def max_over_ranks(value: float, device=None) -> float:
    """Maximum of a per-rank float over the default process group (identity without one)."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(value: float, device=None) -> float:
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())
