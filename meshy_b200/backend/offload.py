"""Colocation hand-off: move a trainer's flat buffers off and back on the GPU.

Reference: ``meshy/backend/titan/trainer.py:327-408`` moves every parameter and
optimiser state with ``Module.to``.  Here the state is five flat buffers, so
offload is five large pinned copies on a side stream, and restore re-points
every parameter view at the new storage.
"""

from __future__ import annotations

import torch

_BUFS = ("master", "grad", "exp_avg", "exp_avg_sq", "compute")


def offload(trainer) -> None:
    offload_flat(trainer.flat)


def restore(trainer) -> None:
    restore_flat(trainer.flat)


def offload_flat(f) -> None:
    """Move every flat buffer of a :class:`~.flat.FlatParams` to pinned host memory."""
    if getattr(f, "sharded", False):
        return f.offload()
    if f.master is None or f.master.device.type != "cuda":
        return
    host = {}
    keep = set(getattr(f, "resident", ()))  # buffers that must stay mapped (symmetric heap)
    for name in _BUFS:
        if name in keep:
            continue
        t = getattr(f, name)
        if t is None or (name == "compute" and not f.separate_compute):
            continue
        h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
        h.copy_(t, non_blocking=True)
        host[name] = h
    torch.cuda.synchronize()
    f._host = host
    for name in host:
        setattr(f, name, None)
    if not keep:
        for p in f.params:
            p.data = torch.empty(0, dtype=p.dtype, device=p.device)
            p.main_grad = None
    torch.cuda.empty_cache()


def restore_flat(f) -> None:
    """Inverse of :func:`offload_flat`: buffers back on the device, parameter views re-pointed."""
    if getattr(f, "sharded", False):
        return f.restore()
    host = getattr(f, "_host", None)
    if not host:
        return
    for name, h in host.items():
        setattr(f, name, h.to(f.device, non_blocking=True))
    if not f.separate_compute:
        f.compute = f.master
    for s, p in zip(f.slots, f.params):
        p.data = f.compute[s.offset:s.offset + s.numel].view(s.shape)
        g = f.grad[s.offset:s.offset + s.numel].view(s.shape)
        if f.separate_compute:
            p.main_grad = g
        else:
            p.grad = g
    torch.cuda.synchronize()
    f._host = None


__all__ = ["offload", "offload_flat", "restore", "restore_flat"]
