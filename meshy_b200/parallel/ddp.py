"""Data-parallel gradient reduction over the flat fp32 gradient buffer.

The reference runs DDP as HSDP with an fp32 gradient all-reduce per FSDP
unit (``TT:torchtitan/models/qwen3/parallelize.py:88-112``; loss already
divided by global denominators, so the reduction is a plain SUM).  Here the
gradient is one flat buffer, so the reduction is a handful of large
collectives:

* within one node with peer access, the fused NVLink kernel
  (:mod:`meshy_b200.parallel.symm` ``all_reduce``): each rank reduces its
  slice straight from every peer's buffer and writes the result back into
  every peer (P2P loads/stores, no staging copy);
* otherwise NCCL ``all_reduce`` on the flat buffer in buckets.
"""

from __future__ import annotations

import os

import torch
import torch.distributed as dist

BUCKET_ELEMS = 64 * 1024 * 1024  # 256 MiB of fp32 per collective


class GradReducer:
    def __init__(self, flat, group=None, *, backend: str | None = None):
        self.flat = flat
        self.group = group
        self.world = dist.get_world_size(group) if (group is not None and dist.is_initialized()) else 1
        self.backend = backend or os.environ.get("MESHY_GRAD_REDUCE", "auto")
        self._symm = None
        self.last_bytes = 0

    def arm(self) -> None:
        """Called before the last micro-batch's backward of a mini-batch."""

    def _fused(self):
        if self._symm is None:
            from .symm import SymmetricAllReduce

            self._symm = SymmetricAllReduce.create(self.flat.grad, self.group)
        return self._symm

    def finish(self) -> None:
        if self.world <= 1:
            return
        g = self.flat.grad
        self.last_bytes = g.numel() * g.element_size()
        use_fused = g.is_cuda and self.backend in ("auto", "fused")
        if use_fused:
            try:
                ar = self._fused()
            except Exception:
                if self.backend == "fused":
                    raise
                ar = None
                self.backend = "nccl"
            if ar is not None:
                ar.all_reduce_()
                return
        for s in range(0, g.numel(), BUCKET_ELEMS):
            dist.all_reduce(g[s:s + BUCKET_ELEMS], group=self.group)


__all__ = ["GradReducer"]
