"""Tensor-parallel rollout engine: one process per GPU, driven in lock-step by rank 0.

The reference gets tensor-parallel inference from SGLang (``tp_size`` in ``meshy/service/inference.py:244-256``).
Here a replica of ``tp`` GPUs runs ``tp`` :class:`~meshy_b200.rollout.engine.RolloutEngine` processes, each
holding its heads and FFN slice of every block (``tp_group``). Rank 0 owns the HTTP server and the scheduler
state that clients see; every engine call that changes state or launches kernels goes through
:class:`EngineLeader`, which first broadcasts the call (name and arguments, over a gloo group) to the followers
(:func:`follow`) and then runs it locally. All ranks therefore admit, prefill and decode the same requests in
the same order, their row-parallel partial sums meet in the same all-reduces, and their samplers draw the same
tokens (the LM head is replicated and the sampling noise is keyed by seed, step and row). Followers drop their
finished generations; only rank 0 answers clients.
"""

from __future__ import annotations

import threading
from typing import Any

import torch.distributed as dist

# engine methods whose calls every rank must make, in the same order
LOCKSTEP = frozenset({
    "submit", "step", "run_until_idle", "generate", "abort_all", "pause", "resume", "release_memory",
    "resume_memory", "update_weights_from_state_dict", "update_weights_from_disk", "update_weights_from_ipc",
})


def _to_host(obj):
    """Tensors in a broadcast call go by value through host memory: a pickled CUDA tensor would be rebuilt on
    rank 0's device in the follower's process."""
    import torch

    if isinstance(obj, torch.Tensor):
        return obj.detach().cpu()
    if isinstance(obj, dict):
        return {k: _to_host(v) for k, v in obj.items()}
    if isinstance(obj, (list, tuple)):
        return type(obj)(_to_host(v) for v in obj)
    return obj


class EngineLeader:
    """Rank 0's engine handle: lock-step calls are broadcast to the followers before they run here; everything
    else (attributes, read-only helpers) is the local engine's."""

    def __init__(self, engine, ctrl_group):
        self._engine = engine
        self._group = ctrl_group
        self._order = threading.RLock()  # one broadcast + local call at a time, in one order for every rank

    def _broadcast(self, obj) -> None:
        dist.broadcast_object_list([_to_host(obj)], src=0, group=self._group)

    def __getattr__(self, name: str) -> Any:
        attr = getattr(self._engine, name)
        if name not in LOCKSTEP or not callable(attr):
            return attr

        def call(*args, **kwargs):
            with self._order:
                self._broadcast((name, args, kwargs))
                return attr(*args, **kwargs)

        return call

    def stop(self) -> None:
        with self._order:
            self._broadcast(("__stop__", (), {}))


def follow(engine, ctrl_group) -> None:
    """A follower rank's loop: run every broadcast call on the local engine until rank 0 stops."""
    while True:
        box = [None]
        dist.broadcast_object_list(box, src=0, group=ctrl_group)
        name, args, kwargs = box[0]
        if name == "__stop__":
            return
        getattr(engine, name)(*args, **kwargs)
        engine.finished.clear()  # only rank 0 answers clients


__all__ = ["EngineLeader", "LOCKSTEP", "follow"]
