"""Host-side helpers for running batches of independent cluster problems on several GPUs.

One process per GPU (torchrun). Batches shard with no inter-GPU traffic: every rank owns a contiguous
range of problems; the only collectives are the host-side timing reductions (max over ranks).
"""
from __future__ import annotations


def shard_range(total, rank, world):
    """Contiguous [start, start + count) of `total` problems owned by `rank` (the first total % world ranks
    get one extra)."""
    if world < 1 or not 0 <= rank < world or total < 0:
        raise ValueError(f"bad shard request total={total} rank={rank} world={world}")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def max_over_ranks(value, dist=None, device=None):
    """Max of a float over all ranks (identity without a process group)."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    import torch

    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(value, dist=None, device=None):
    """Sum of a number over all ranks (identity without a process group)."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    import torch

    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())
