"""Run artifact layout (``weights/``, ``state/``, ``logs/``, ``tensorboard/``,
``trajectories.jsonl``) with ``XRL_*`` overrides, plus readiness markers kept
in the bootstrap store (reference ``meshy/service/runtime.py:26-135``)."""

from __future__ import annotations

import os

from . import bootstrap


class RuntimeDir:
    def __init__(self, root: str, *, checkpoint_dir=None, log_dir=None, tensorboard_dir=None, trajectory_dir=None,
                 state_dir=None):
        self.root = os.path.abspath(root)
        os.makedirs(self.root, exist_ok=True)
        env = os.environ.get
        self.checkpoint_dir = os.path.abspath(checkpoint_dir or env("XRL_CHECKPOINT_DIR")
                                              or os.path.join(self.root, "weights"))
        self.state_dir = os.path.abspath(state_dir or env("XRL_STATE_DIR") or os.path.join(self.root, "state"))
        self.log_dir = os.path.abspath(log_dir or env("XRL_LOG_DIR") or os.path.join(self.root, "logs"))
        self.tensorboard_dir = os.path.abspath(tensorboard_dir or env("XRL_TENSORBOARD_DIR")
                                               or os.path.join(self.root, "tensorboard"))
        self.trajectory_dir = os.path.abspath(trajectory_dir or env("XRL_TRAJECTORY_DIR") or self.root)

    @classmethod
    def from_env(cls, default_root: str | None = None) -> "RuntimeDir":
        return cls(os.environ.get("XRL_RUNTIME_DIR") or default_root or os.path.join(".xrl_runtime", "default"))

    def process_log_path(self, service_name: str, rank_in_service: int) -> str:
        os.makedirs(self.log_dir, exist_ok=True)
        return os.path.join(self.log_dir, f"{service_name}-{int(rank_in_service)}.log")

    def checkpoint_path(self, service_name: str, version: int) -> str:
        return os.path.join(self.checkpoint_dir, service_name, f"v{int(version)}")

    def weights_dir(self, service_name: str) -> str:
        return os.path.join(self.checkpoint_dir, service_name)

    def state_store(self):
        from .checkpoint import StateStore

        return StateStore(self.state_dir)

    def tensorboard_path(self, service_name: str) -> str:
        return os.path.join(self.tensorboard_dir, service_name)

    def trajectory_path(self) -> str:
        return os.path.join(self.trajectory_dir, "trajectories.jsonl")

    def _ready_key(self, name: str) -> str:
        return f"ready|{self.root}|{name}"

    def mark_ready(self, name: str) -> None:
        bootstrap.mark(self._ready_key(name))

    def is_ready(self, name: str) -> bool:
        return bootstrap.check([self._ready_key(name)])

    def wait_ready(self, names, timeout: float = 1800.0, interval: float = 1.0, liveness=None) -> None:
        pending = list(dict.fromkeys(names))
        if not pending:
            return
        try:
            bootstrap.wait_keys([self._ready_key(n) for n in pending], timeout=timeout, interval=interval,
                                liveness=liveness)
        except TimeoutError:
            missing = [n for n in pending if not self.is_ready(n)]
            raise TimeoutError(f"services never became ready: {missing}") from None


__all__ = ["RuntimeDir"]
