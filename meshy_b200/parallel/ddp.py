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
* otherwise NCCL ``all_reduce`` of the flat buffer, overlapped with the
  backward: during the last micro-batch of a mini-batch (:meth:`GradReducer.arm`)
  each transformer block's gradient range is summed by an asynchronous
  all-reduce as soon as that block's backward has been issued (a
  :class:`~meshy_b200.parallel.fsdp.BlockBoundary` at the block's input
  reports it), while the earlier blocks' backward runs; :meth:`GradReducer.finish`
  waits for them and sums the rest (embedding, final norm, LM head) in
  buckets. Every rank's backward visits the blocks in the same order, so the
  collectives match across ranks. ``MESHY_DDP_OVERLAP=0`` keeps everything
  for :meth:`finish`.
"""

from __future__ import annotations

import os

import torch
import torch.distributed as dist

BUCKET_ELEMS = 64 * 1024 * 1024  # 256 MiB of fp32 per collective


def _subtract(lo: int, hi: int, holes: list[tuple[int, int]]):
    """``[lo, hi)`` minus the sorted, disjoint ``holes`` ``(start, end)``."""
    pos = lo
    for a, b in holes:
        if b <= pos or a >= hi:
            continue
        if a > pos:
            yield pos, a
        pos = max(pos, b)
    if pos < hi:
        yield pos, hi


class GradReducer:
    """``skip`` lists ``(offset, numel)`` ranges of the flat gradient that must not be summed over
    ``group`` (expert-parallel experts: every rank holds different experts).

    It also serves as the model's block hooks (``DecoderLM.block_hooks``: ``begin_forward``, ``pre_block``,
    ``post_block``, ``backward_begin``, ``backward_end``) for the overlapped reduction."""

    def __init__(self, flat, group=None, *, backend: str | None = None, skip: list[tuple[int, int]] | None = None,
                 overlap: bool | None = None):
        self.flat = flat
        self.group = group
        self.world = dist.get_world_size(group) if (group is not None and dist.is_initialized()) else 1
        self.backend = backend or os.environ.get("MESHY_GRAD_REDUCE", "auto")
        self.last_bytes = 0
        self.skip = sorted(skip or [])
        self._holes = [(o, o + n) for o, n in self.skip]
        self.overlap = overlap if overlap is not None else os.environ.get("MESHY_DDP_OVERLAP", "1") != "0"
        self._blocks = self._block_ranges()
        self._armed = False
        self._works: list = []
        self._done: list[tuple[int, int]] = []

    def _block_ranges(self) -> dict[int, tuple[int, int, list]]:
        """Block index -> (lo, hi, [(slot, param)]) for every block whose parameters are contiguous in the
        flat layout (``layers.<i>.*``; the flat buffer is laid out in ``named_parameters`` order)."""
        out: dict[int, tuple[int, int, list]] = {}
        slots = getattr(self.flat, "slots", None)
        params = getattr(self.flat, "params", None)
        if not slots or params is None or getattr(self.flat, "sharded", False):
            return out
        members: dict[int, list] = {}
        for s, p in zip(slots, params):
            parts = s.name.split(".")
            if len(parts) > 2 and parts[0] == "layers" and parts[1].isdigit():
                members.setdefault(int(parts[1]), []).append((s, p))
        for i, mem in members.items():
            lo = min(s.offset for s, _ in mem)
            hi = max(s.offset + s.numel for s, _ in mem)
            if hi - lo == sum(s.numel for s, _ in mem):
                out[i] = (lo, hi, mem)
        return out

    @property
    def overlapping(self) -> bool:
        """Whether the block hooks launch reductions during the armed backward."""
        return self.overlap and self.world > 1 and self.backend != "none" and bool(self._blocks)

    def _ranges(self, n: int):
        yield from _subtract(0, n, self._holes)

    # ------------------------------------------------------------------ block hooks
    def begin_forward(self) -> None:
        pass

    def pre_block(self, i: int, x: torch.Tensor) -> torch.Tensor:
        if self.overlapping and torch.is_grad_enabled() and x.requires_grad:
            from .fsdp import BlockBoundary

            x = BlockBoundary.apply(x, self, i, "in")
        return x

    def post_block(self, i: int, x: torch.Tensor) -> torch.Tensor:
        return x

    def backward_begin(self, i: int) -> None:
        pass

    def backward_end(self, i: int) -> None:
        """Block ``i``'s backward is issued: its gradient is final for this mini-batch, so sum it now."""
        if not self._armed or i not in self._blocks:
            return
        lo, hi, mem = self._blocks[i]
        if getattr(self.flat, "separate_compute", False):  # PyTorch paths: fold this block's .grad first
            with torch.no_grad():
                for _s, p in mem:
                    if p.grad is not None:
                        p.main_grad.add_(p.grad)
                        p.grad = None
        g = self.flat.grad
        for a, b in _subtract(lo, hi, self._holes):
            part = g[a:b]
            self.last_bytes += part.numel() * part.element_size()
            self._works.append(dist.all_reduce(part, group=self.group, async_op=True))
        self._done.append((lo, hi))

    # ------------------------------------------------------------------ step
    def arm(self) -> None:
        """Called before the last micro-batch's backward of a mini-batch."""
        self.last_bytes = 0
        self._works, self._done = [], []
        self._armed = self.overlapping

    def finish(self) -> None:
        armed, self._armed = self._armed, False
        if self.world <= 1 or self.backend == "none":
            return
        if not armed:
            self.last_bytes = 0
        for w in self._works:
            w.wait()
        done = sorted(self._done)
        self._works, self._done = [], []
        g = self.flat.grad
        for lo, hi in self._ranges(g.numel()):
            for a, b in _subtract(lo, hi, done):
                for s in range(a, b, BUCKET_ELEMS):
                    part = g[s:min(b, s + BUCKET_ELEMS)]
                    self.last_bytes += part.numel() * part.element_size()
                    dist.all_reduce(part, group=self.group)


__all__ = ["GradReducer"]
