"""Session sharding across GPUs (one process per GPU).

Needle-3 sessions are independent (crates/needle-infer/src/v3_engine.rs:543-560:
each call owns its V3Cache, weights are immutable), so a serving job splits its
sessions into contiguous ranges, one per rank, replicates the container on every
GPU and runs with no collective on the data path. The only cross-rank steps are
the timing barrier and the max-over-ranks reduction of the device time.
"""
from __future__ import annotations


def session_range(total: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of the sessions owned by `rank`: contiguous ranges whose
    sizes differ by at most one (the first total % world ranks take one more)."""
    if world <= 0 or not 0 <= rank < world or total < 0:
        raise ValueError("need world > 0, 0 <= rank < world and total >= 0")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def max_over_ranks(value: float, dist=None, device=None) -> float:
    """The maximum of `value` over all ranks of the default process group (the
    value itself when `dist` is None or the group has one rank)."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    import torch
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
