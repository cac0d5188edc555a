"""Where a run keeps its artifacts, and how its services announce readiness.

A run owns one root directory. Each artifact kind lives in a subdirectory
unless the launcher flag or an ``XRL_*`` variable points it elsewhere (these
variable names and the default layout are the user-facing contract of the
reference, ``meshy/service/runtime.py:26-135``)::

    <root>/weights/<service>/v<version>/    HF safetensors exports
    <root>/state/<service>/step-<n>...       global checkpoints (StateStore)
    <root>/logs/<service>-<rank>.log         per-process logs
    <root>/tensorboard/<service>/            metric events
    <root>/trajectories.jsonl                rollout trajectories

Readiness is not a file: a service marks ``ready|<root>|<name>`` in the
bootstrap key-value store (:mod:`.bootstrap`), so waiting on it needs no
shared filesystem and the markers of an older run under the same root are
never seen by a new launch (the store lives as long as the launcher).
"""

from __future__ import annotations

import os
from typing import Callable, Iterable

from . import bootstrap

# artifact kind -> (constructor keyword, environment override, default location under the root;
# None means the root itself)
_LOCATIONS = {
    "checkpoint_dir": ("XRL_CHECKPOINT_DIR", "weights"),
    "state_dir": ("XRL_STATE_DIR", "state"),
    "log_dir": ("XRL_LOG_DIR", "logs"),
    "tensorboard_dir": ("XRL_TENSORBOARD_DIR", "tensorboard"),
    "trajectory_dir": ("XRL_TRAJECTORY_DIR", None),
}

DEFAULT_ROOT = os.path.join(".xrl_runtime", "default")


class RuntimeDir:
    """Resolved artifact locations of one run (explicit argument > ``XRL_*`` variable > default)."""

    def __init__(self, root: str, **overrides: str | None):
        unknown = set(overrides) - set(_LOCATIONS)
        if unknown:
            raise TypeError(f"unknown runtime locations: {sorted(unknown)}")
        self.root = os.path.abspath(root)
        os.makedirs(self.root, exist_ok=True)
        for kind, (env, sub) in _LOCATIONS.items():
            chosen = overrides.get(kind) or os.environ.get(env)
            if not chosen:
                chosen = os.path.join(self.root, sub) if sub else self.root
            setattr(self, kind, os.path.abspath(chosen))

    @classmethod
    def from_env(cls, default_root: str | None = None) -> "RuntimeDir":
        """The run of this process: ``XRL_RUNTIME_DIR`` (set by the launcher), else ``default_root``."""
        return cls(os.environ.get("XRL_RUNTIME_DIR") or default_root or DEFAULT_ROOT)

    # ------------------------------------------------------------------ paths
    def process_log_path(self, service_name: str, rank_in_service: int) -> str:
        os.makedirs(self.log_dir, exist_ok=True)
        return os.path.join(self.log_dir, "%s-%d.log" % (service_name, int(rank_in_service)))

    def weights_dir(self, service_name: str) -> str:
        return os.path.join(self.checkpoint_dir, service_name)

    def checkpoint_path(self, service_name: str, version: int) -> str:
        """Directory of the HF export of weight version ``version``."""
        return os.path.join(self.weights_dir(service_name), "v%d" % int(version))

    def tensorboard_path(self, service_name: str) -> str:
        return os.path.join(self.tensorboard_dir, service_name)

    def trajectory_path(self) -> str:
        return os.path.join(self.trajectory_dir, "trajectories.jsonl")

    def state_store(self):
        from .checkpoint import StateStore

        return StateStore(self.state_dir)

    # ------------------------------------------------------------------ readiness
    def _marker(self, name: str) -> str:
        return "|".join(("ready", self.root, name))

    def mark_ready(self, name: str) -> None:
        bootstrap.mark(self._marker(name))

    def is_ready(self, name: str) -> bool:
        return bootstrap.check([self._marker(name)])

    def wait_ready(self, names: Iterable[str], timeout: float = 1800.0, interval: float = 1.0,
                   liveness: Callable[[], bool] | None = None) -> None:
        """Block until every named service is ready; a failed ``liveness`` probe or the timeout raises."""
        wanted: list[str] = []
        for n in names:
            if n not in wanted:
                wanted.append(n)
        if not wanted:
            return
        try:
            bootstrap.wait_keys([self._marker(n) for n in wanted], timeout=timeout, interval=interval,
                                liveness=liveness)
        except TimeoutError:
            late = [n for n in wanted if not self.is_ready(n)]
            raise TimeoutError("still waiting for %s after %.0f s" % (", ".join(late), timeout)) from None


__all__ = ["DEFAULT_ROOT", "RuntimeDir"]
