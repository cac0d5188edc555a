"""Accumulating named stopwatches (reference ``meshy/utils/timer.py:53-178``).

``TimerStats.timer(name, sync=...)`` accumulates time per bucket.  On a CUDA
machine every bucket is device time: a pair of CUDA events on the current
stream brackets the block, and :meth:`TimerStats.pop_metrics` waits for the
last event once and sums the elapsed times, so timing adds no host sync inside
the step.  ``sync=True`` additionally brackets the block with
``torch.cuda.synchronize`` (the bucket then also covers host work that kept
the device idle).  On CPU the buckets are wall time.
:class:`DeviceTimer` times a region with CUDA events instead (no host sync
inside the region); :func:`max_over_ranks` turns a per-rank time into the
job time. Every timed region, and every :func:`nvtx_range`, is also an NVTX
range on a CUDA machine (``MESHY_NVTX=0`` turns them off), so a profiler
timeline (or ``ncu --nvtx --nvtx-include``) shows the RL step's phases.
"""

from __future__ import annotations

import os
import time
from collections import defaultdict
from contextlib import contextmanager

import torch

_GLOBAL_ENABLED = True


_NVTX_BROKEN = False


def _nvtx_on() -> bool:
    return (not _NVTX_BROKEN and os.environ.get("MESHY_NVTX", "1") != "0" and torch.cuda.is_available()
            and torch.cuda.is_initialized())


@contextmanager
def nvtx_range(name: str):
    """An NVTX range around the block on a CUDA machine (a no-op otherwise, or if NVTX is unavailable)."""
    global _NVTX_BROKEN
    pushed = False
    if _nvtx_on():
        try:
            torch.cuda.nvtx.range_push(name)
            pushed = True
        except Exception:  # profiling annotations must never fail the step
            _NVTX_BROKEN = True
    try:
        yield
    finally:
        if pushed:
            torch.cuda.nvtx.range_pop()


def set_timers_enabled(flag: bool) -> None:
    global _GLOBAL_ENABLED
    _GLOBAL_ENABLED = bool(flag)


def _cuda_live() -> bool:
    return torch.cuda.is_available() and torch.cuda.is_initialized()


class TimerStats:
    def __init__(self, enabled: bool = True, device: bool | None = None):
        self.enabled = enabled
        self.device = device
        self.totals: dict[str, float] = defaultdict(float)
        self.counts: dict[str, int] = defaultdict(int)
        self._events: list[tuple[str, object, object]] = []

    @contextmanager
    def timer(self, name: str, sync: bool = False):
        if not (self.enabled and _GLOBAL_ENABLED):
            with nvtx_range(name):
                yield
            return
        cuda = _cuda_live() and (self.device is None or self.device)
        if cuda and torch.cuda.is_current_stream_capturing():
            cuda = sync = False  # events cannot be timed inside a graph capture
        if cuda and sync:
            torch.cuda.synchronize()
        t0 = time.perf_counter()
        ev = None
        if cuda:
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ev[0].record()
        try:
            with nvtx_range(name):
                yield
        finally:
            if ev is not None:
                ev[1].record()
                if sync:
                    torch.cuda.synchronize()
                self._events.append((name, ev[0], ev[1]))
            else:
                self.totals[name] += time.perf_counter() - t0
            self.counts[name] += 1

    def add(self, name: str, seconds: float) -> None:
        self.totals[name] += seconds
        self.counts[name] += 1

    def _drain(self) -> None:
        if not self._events:
            return
        self._events[-1][2].synchronize()
        for name, s, e in self._events:
            e.synchronize()
            self.totals[name] += s.elapsed_time(e) / 1e3
        self._events.clear()

    def pop_metrics(self, prefix: str = "") -> dict[str, float]:
        self._drain()
        out = {f"{prefix}{k}": v for k, v in self.totals.items()}
        self.totals.clear()
        self.counts.clear()
        return out


class DeviceTimer:
    """CUDA-event timer on the current stream: ``start()`` … ``stop()`` → ms."""

    def __init__(self):
        self._s = torch.cuda.Event(enable_timing=True)
        self._e = torch.cuda.Event(enable_timing=True)

    def start(self):
        self._s.record()
        return self

    def stop(self) -> float:
        self._e.record()
        self._e.synchronize()
        return self._s.elapsed_time(self._e)


def max_over_ranks(value: float, group=None, device=None) -> float:
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size(group) == 1:
        return value
    backend = dist.get_backend(group)
    dev = device if device is not None else (torch.device("cuda") if backend == "nccl" else torch.device("cpu"))
    t = torch.tensor([value], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


__all__ = ["DeviceTimer", "TimerStats", "max_over_ranks", "nvtx_range", "set_timers_enabled"]
