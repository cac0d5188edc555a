"""Data-parallel gradient reduction over the flat fp32 gradient buffer.

The reference runs DDP as HSDP with an fp32 gradient all-reduce per FSDP
unit (``TT:torchtitan/models/qwen3/parallelize.py:88-112``; loss already
divided by global denominators, so the reduction is a plain SUM).  Here the
gradient is one flat buffer, so the reduction is a handful of large
collectives:

* within one node the trainer normally skips this class: the fused NVLink
  optimiser (:class:`meshy_b200.parallel.symm.FusedDPAdamW`) reduces,
  clips, updates and all-gathers in one device pipeline (backend ``none``
  here);
* otherwise NCCL ``all_reduce`` on the flat buffer in buckets.
"""

from __future__ import annotations

import os

import torch
import torch.distributed as dist

BUCKET_ELEMS = 64 * 1024 * 1024  # 256 MiB of fp32 per collective


class GradReducer:
    """``skip`` lists ``(offset, numel)`` ranges of the flat gradient that must not be summed over
    ``group`` (expert-parallel experts: every rank holds different experts)."""

    def __init__(self, flat, group=None, *, backend: str | None = None, skip: list[tuple[int, int]] | None = None):
        self.flat = flat
        self.group = group
        self.world = dist.get_world_size(group) if (group is not None and dist.is_initialized()) else 1
        self.backend = backend or os.environ.get("MESHY_GRAD_REDUCE", "auto")
        self.last_bytes = 0
        self.skip = sorted(skip or [])

    def _ranges(self, n: int):
        pos = 0
        for off, cnt in self.skip:
            if off > pos:
                yield pos, off
            pos = max(pos, off + cnt)
        if pos < n:
            yield pos, n

    def arm(self) -> None:
        """Called before the last micro-batch's backward of a mini-batch."""

    def finish(self) -> None:
        if self.world <= 1 or self.backend == "none":
            return
        g = self.flat.grad
        self.last_bytes = 0
        for lo, hi in self._ranges(g.numel()):
            for s in range(lo, hi, BUCKET_ELEMS):
                part = g[s:min(hi, s + BUCKET_ELEMS)]
                self.last_bytes += part.numel() * part.element_size()
                dist.all_reduce(part, group=self.group)


__all__ = ["GradReducer"]
