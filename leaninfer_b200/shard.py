"""Sequence sharding across ranks (one process per GPU).

Decode sequences are independent: each carries its own recurrent state and
conv state, and a layer step for one sequence reads nothing of another. A
global batch therefore splits into contiguous per-rank ranges with no data
exchange during the step; the only collective is the max-reduction of the
measured time. The layer weights are replicated on every rank.
"""
from __future__ import annotations


def shard_bounds(n_total: int, world: int, rank: int) -> tuple[int, int]:
    """(first, count) of rank's contiguous range of n_total sequences; the
    first n_total % world ranks take one more."""
    if world <= 0 or not 0 <= rank < world or n_total < 0:
        raise ValueError(f"bad shard request n_total={n_total} world={world} rank={rank}")
    base, extra = divmod(n_total, world)
    count = base + (1 if rank < extra else 0)
    first = rank * base + min(rank, extra)
    return first, count


def max_over_ranks(values, dist=None, device=None) -> list[float]:
    """Element-wise maximum of per-rank float values (identity without a
    process group); every rank must call it with the same length."""
    vals = [float(v) for v in values]
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return vals
    import torch
    t = torch.tensor(vals, dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(x) for x in t.tolist()]
