"""Token sharding of MhcPre across GPUs (one process per GPU).

Rows (tokens) are independent, so the work shards without any collective on the
data path: rank r of W takes the contiguous rows shard_range(M, W, r) (ceil-div
shards, the last ones smaller or empty), phi/gamma/alpha/bias are replicated and
prepared on every GPU.  From 8192 rows per shard up, the split-K plan depends on K
only, so every row's result bits equal the unsharded run's.

Collectives are used only around the hot path: gather_outputs() collects the
shards' outputs (for validation), and max_over_ranks() takes the slowest rank's
time.  Both work with any torch.distributed backend (nccl on GPUs, gloo on CPU).
"""
from __future__ import annotations


def shard_range(M: int, world: int, rank: int) -> tuple[int, int]:
    """(first row, row count) of rank's contiguous shard of M rows."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    per = -(-M // world)
    start = min(rank * per, M)
    return start, min(per, M - start)


def gather_outputs(local, M: int, group=None):
    """All-gathers per-rank output shards along dim 0 into full [M, ...] tensors.

    local: tensors whose dim 0 is this rank's row count (shard_range order).
    Shards are padded to the largest shard size for the collective, then trimmed.
    Returns the full tensors on every rank."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    per = -(-M // world)
    full = []
    for t in local:
        padded = t.new_zeros((per,) + tuple(t.shape[1:]))
        if t.shape[0]:
            padded[: t.shape[0]].copy_(t)
        parts = [torch.empty_like(padded) for _ in range(world)]
        if t.element_size() == 2:
            # a gather is a copy: move 16-bit elements as bytes (gloo has no 16-bit types)
            dist.all_gather([p.view(torch.uint8) for p in parts], padded.view(torch.uint8), group=group)
        else:
            dist.all_gather(parts, padded, group=group)
        rows = [shard_range(M, world, r)[1] for r in range(world)]
        full.append(torch.cat([p[:n] for p, n in zip(parts, rows)], dim=0))
    return tuple(full)


def max_over_ranks(value: float, group=None, device=None) -> float:
    """The largest value over all ranks (e.g. a per-rank device time)."""
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
