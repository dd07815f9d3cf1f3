"""Data parallelism over independent sequences (one process per GPU, no data-path collective).

Sequences are split into contiguous blocks, one per rank; each rank decodes its block
with its own weight replica, slot caches and eviction state.  Collectives are used only
for bookkeeping: gathering per-sequence results and taking the max of per-rank timings.
"""

from __future__ import annotations

from typing import Any, Callable, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist


def shard_range(n: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous block [lo, hi) of ``n`` items for ``rank`` of ``world`` (sizes differ by <= 1)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def run_data_parallel(
    generate_fn: Callable[[Sequence[Sequence[int]]], List[Any]],
    batch_input_ids: Sequence[Sequence[int]],
    group: Optional[dist.ProcessGroup] = None,
) -> List[Any]:
    """Decode this rank's shard with ``generate_fn`` and return every rank's results in
    global sequence order (on every rank)."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    lo, hi = shard_range(len(batch_input_ids), rank, world)
    mine = generate_fn(batch_input_ids[lo:hi]) if hi > lo else []
    if world == 1:
        return list(mine)
    parts: List[Any] = [None] * world
    dist.all_gather_object(parts, list(mine), group=group)
    out: List[Any] = []
    for p in parts:
        out.extend(p)
    return out


def max_over_ranks(value: float, device: Optional[torch.device] = None, group=None) -> float:
    """Max of a per-rank scalar (e.g. a device-timed duration) over all ranks."""
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device or "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
