"""Service / ServiceGroup abstractions and process utilities.

A :class:`ServiceGroup` declares a group of engine replicas (role config,
replica count, cards per replica, ``colocate_with``, ``wait_until``); the
:class:`~meshy_b200.service.ignite.Ignitor` expands groups into per-card
:class:`Service` objects whose ``ignite()`` starts the role's engine process
and ``wait_for_ready()`` publishes readiness.  Same contract as the reference
(``meshy/service/base.py:37-276``).  Import-light: no torch here, so a
launcher can read a recipe cheaply.
"""

from __future__ import annotations

import os
import sys
from dataclasses import dataclass, field
from typing import TYPE_CHECKING, Any

from ..config import ServiceConfig

if TYPE_CHECKING:
    from .runtime import RuntimeDir
    from .topology import ServiceInfo, Topology


def die_with_parent(signal_number: int | None = None) -> None:
    """``PR_SET_PDEATHSIG``: the kernel kills this process when its parent dies."""
    import platform
    import signal

    if platform.system() != "Linux":
        return
    try:
        import ctypes

        ctypes.CDLL("libc.so.6", use_errno=True).prctl(1, signal.SIGKILL if signal_number is None else signal_number)
    except Exception:
        pass


def raise_open_file_limit() -> int:
    """Raise the soft ``RLIMIT_NOFILE`` to the hard limit; returns the new soft limit or -1."""
    try:
        import resource

        soft, hard = resource.getrlimit(resource.RLIMIT_NOFILE)
        if hard != resource.RLIM_INFINITY and soft >= hard:
            return soft
        resource.setrlimit(resource.RLIMIT_NOFILE, (hard, hard))
        return resource.getrlimit(resource.RLIMIT_NOFILE)[0]
    except Exception:
        return -1


def redirect_output(log_path: str) -> None:
    """Point fds 1 and 2 at an append-only log (captures native output too)."""
    d = os.path.dirname(os.path.abspath(log_path))
    os.makedirs(d, exist_ok=True)
    fd = os.open(log_path, os.O_WRONLY | os.O_CREAT | os.O_APPEND, 0o644)
    for s in (sys.stdout, sys.stderr):
        try:
            s.flush()
        except Exception:
            pass
    os.dup2(fd, 1)
    os.dup2(fd, 2)
    os.close(fd)
    for s in (sys.stdout, sys.stderr):
        try:
            s.reconfigure(line_buffering=True)
        except Exception:
            pass


@dataclass(frozen=True)
class GPU:
    """One physical card as seen by the run (all-gathered at startup)."""

    global_rank: int
    host: str
    local_rank: int
    node_rank: int = 0
    uuid: str = ""


@dataclass
class ServiceGroup:
    id: str
    n_replicas: int
    n_gpus_per_replica: int
    config: ServiceConfig
    colocate_with: str | None = None
    wait_until: list[str] = field(default_factory=list)

    def __post_init__(self) -> None:
        if not self.id:
            raise ValueError("ServiceGroup.id must be non-empty")
        if self.n_replicas <= 0:
            raise ValueError(f"group {self.id!r}: n_replicas must be positive")
        if self.uses_gpu and self.n_gpus_per_replica <= 0:
            raise ValueError(f"GPU group {self.id!r} needs n_gpus_per_replica > 0")
        if not self.uses_gpu and self.n_gpus_per_replica != 0:
            raise ValueError(f"CPU group {self.id!r} must have n_gpus_per_replica == 0")
        if self.colocate_with == self.id:
            raise ValueError(f"group {self.id!r} cannot colocate with itself")

    @property
    def role(self) -> str:
        return type(self.config).role

    @property
    def uses_gpu(self) -> bool:
        return type(self.config).uses_gpu

    @property
    def n_cards(self) -> int:
        return self.n_replicas * self.n_gpus_per_replica if self.uses_gpu else 0


class Service:
    """Runtime entity of one replica inside one ignitor process."""

    def __init__(self, info: "ServiceInfo", topology: "Topology", runtime: "RuntimeDir"):
        self.info = info
        self.topology = topology
        self.runtime = runtime
        self.proc = None
        self.colocation_manager = None

    @classmethod
    def from_info(cls, info: "ServiceInfo", topology: "Topology", runtime: "RuntimeDir") -> "Service":
        return cls(info, topology, runtime)

    @property
    def name(self) -> str:
        return self.info.name

    def configure_colocation(self) -> None:
        """Hook: services in a colocation ring build their ring manager here."""

    def ignite(self) -> None:
        raise NotImplementedError

    def is_alive(self) -> bool:
        return self.proc is not None and self.proc.is_alive() if hasattr(self.proc, "is_alive") else \
            (self.proc is not None and self.proc.poll() is None)

    def wait_for_ready(self, timeout: float = 1800.0) -> None:
        self.runtime.mark_ready(self.name)

    def join(self) -> int:
        if self.proc is None:
            return 0
        if hasattr(self.proc, "join"):
            self.proc.join()
            return self.proc.exitcode or 0
        return self.proc.wait()

    def terminate(self) -> None:
        if self.proc is None:
            return
        try:
            self.proc.terminate()
        except Exception:
            pass

    def health_info(self) -> dict[str, Any]:
        return {"name": self.name, "alive": self.is_alive()}


__all__ = ["GPU", "Service", "ServiceGroup", "die_with_parent", "raise_open_file_limit", "redirect_output"]
