"""Data-parallel plumbing for independent sequences: one process per GPU.

Decode of independent sequences has no exchange step, so the data path uses
no collective; torch.distributed only carries the barrier around the timed
region and the max-over-ranks reduction of the measured time.
"""
from __future__ import annotations

import os


def dist_env() -> tuple[int, int, int]:
    """(rank, world_size, local_rank) from the torchrun environment."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


def shard(n_seq: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous balanced split of n_seq sequences: (first, count) for `rank`."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    base, extra = divmod(n_seq, world)
    count = base + (1 if rank < extra else 0)
    first = rank * base + min(rank, extra)
    return first, count


def max_over_ranks(value: float, device=None) -> float:
    """Max of a per-rank float over the default process group (identity when
    torch.distributed is not initialised)."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()):
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device or "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(value: float, device=None) -> float:
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()):
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device or "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())
