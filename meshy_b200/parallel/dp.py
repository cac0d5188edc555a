"""Data-parallel scatter of a rollout window (reference ``meshy/backend/titan/parallel.py:21-107``).

Rank ``src`` holds the whole window; it is broadcast over the (CPU) control
group and every rank runs the same deterministic planner on the same list,
so each knows its own share without any plan being communicated.  DP ranks
get disjoint subsets (token-balanced by the planner); ranks of one CP or TP
group get the same subset (CP splits sequences later, TP needs identical
inputs).
"""

from __future__ import annotations

from typing import Any, Callable, Sequence

import torch.distributed as dist


def dp_rank_and_size(parallel_dims) -> tuple[int, int]:
    if parallel_dims is None:
        return 0, 1
    return parallel_dims.dp_rank, parallel_dims.dp


def split_batch_to_local(full_batch: Sequence[Any] | None, parallel_dims, group=None, src: int = 0,
                         planner: Callable[[list, int], Any] | None = None):
    """Returns ``(local_samples, local_plan)``; identical within a CP/TP group, disjoint across DP."""
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        box = [list(full_batch) if dist.get_rank() == src else None]
        dist.broadcast_object_list(box, src=src, group=group)
        batch = box[0]
    else:
        batch = list(full_batch)
    if batch is None:
        raise RuntimeError("split_batch_to_local: the source rank held no batch")
    dp_rank, dp_size = dp_rank_and_size(parallel_dims)
    if planner is not None:
        plan = planner(batch, dp_size)
        return plan.local_samples(batch, dp_rank), plan.per_rank[dp_rank]
    if len(batch) % dp_size:
        raise ValueError(f"batch of {len(batch)} is not divisible by the DP size {dp_size}; make rollout batch x "
                         "group size a multiple of dp_replicate x dp_shard")
    n = len(batch) // dp_size
    return batch[dp_rank * n:(dp_rank + 1) * n], None


__all__ = ["dp_rank_and_size", "split_batch_to_local"]
