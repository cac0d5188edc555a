"""SPMD service template: one engine child process per card of a replica.

Same lifecycle contract as the reference (``meshy/service/spmd.py:34-163``):

* ``ignite()`` spawns the child (``spawn`` start method, so no CUDA state or
  threads leak in from the ignitor);
* the child redirects its output to ``logs/<service>-<rank>.log``, arms
  ``PR_SET_PDEATHSIG``, builds the role's engine, joins the replica's process
  groups, builds the colocation manager (rank 0 of the replica only), builds
  the worker, and then either drives (rank 0: the worker's TQ loop submits
  SPMD commands) or follows (ranks > 0: the engine command loop);
* ``wait_for_ready()`` blocks on the child's readiness event while checking
  that it is still alive, then publishes the readiness marker.

Roles subclass :class:`SpmdService` and implement :meth:`build_engine` and
:meth:`build_worker` (both run in the child).
"""

from __future__ import annotations

import logging
import multiprocessing
import os
import time
from typing import Any

from .base import GPU, Service, die_with_parent, redirect_output

log = logging.getLogger(__name__)


def require_ring(info) -> None:
    """A colocated GPU service must be a member of a colocation ring (no silent OOM hours later)."""
    if info.is_colocate and info.colocation is None:
        raise ValueError(
            f"service group {info.group_id!r} shares cards (colocate_with) but is not a member of any "
            "COLOCATIONS ring; declare a ColocationRing covering it and pass it to Ignitor(SERVICE_GROUPS, "
            "COLOCATIONS)")


def current_rank() -> int:
    return int(os.environ.get("RANK", "0"))


class SpmdService(Service):
    """Per-card wrapper of one SPMD replica (trainer, critic, teacher)."""

    def __init__(self, info, topology, runtime, my_gpu: GPU | None = None):
        super().__init__(info, topology, runtime)
        ranks = [g.global_rank for g in info.replica_gpus]
        rank = current_rank() if my_gpu is None else my_gpu.global_rank
        if rank not in ranks:
            raise ValueError(f"rank {rank} is not a card of {info.name} ({ranks})")
        self.my_gpu = info.replica_gpus[ranks.index(rank)]
        self.rank_in_replica = ranks.index(rank)
        self.world_size = len(ranks)
        self.is_master = self.rank_in_replica == 0
        self.processes: list = []
        self._ready = None
        self._error = None

    @classmethod
    def from_info(cls, info, topology, runtime, my_gpu: GPU | None = None) -> "SpmdService":
        return cls(info, topology, runtime, my_gpu)

    # ── role hooks (child process) ──────────────────────────────────────────
    @property
    def device(self) -> str:
        cfg = self.info.config
        dev = getattr(cfg, "device", None) or os.environ.get("XRL_DEVICE", "cuda")
        return f"cuda:{self.my_gpu.local_rank}" if dev == "cuda" else dev

    def engine_kwargs(self) -> dict[str, Any]:
        return dict(rank=self.rank_in_replica, world_size=self.world_size, master_addr=self.info.host,
                    master_port=self.info.dist_port, device=self.device)

    def build_engine(self):  # pragma: no cover - interface
        raise NotImplementedError

    def build_worker(self, engine, colocation):  # pragma: no cover - interface
        raise NotImplementedError

    def build_colocation_manager(self, engine):
        """Ring manager of this replica (rank 0 only); None outside a ring."""
        ring = self.info.colocation
        if ring is None or not self.is_master:
            return None
        from .colocation import ColocationManager

        return ColocationManager(ring, self.info.group_id, self._ledger_factory(ring),
                                 on_acquire=getattr(engine, "on_colocate_acquire", None),
                                 on_release=getattr(engine, "on_colocate_release", None))

    def _ledger_factory(self, ring):
        from ..tq.client import connect
        from .colocation import StoreLedger
        from ..utils.faults import inject

        ref = self.runtime_tq_ref()
        return lambda: inject(StoreLedger(connect(ref), ring.group_id), "ledger")

    def runtime_tq_ref(self) -> str | None:
        cfg = self.info.config
        return getattr(cfg, "tq_endpoints_file", None) or os.environ.get("XRL_TQ_ENDPOINTS")

    # ── lifecycle ───────────────────────────────────────────────────────────
    def ignite(self) -> None:
        ctx = multiprocessing.get_context("spawn")
        self._ready = ctx.Event()
        self._error = ctx.Queue()
        p = ctx.Process(target=self._run_runtime, name=f"{self.name}-{self.rank_in_replica}", daemon=False)
        p.start()
        self.proc = p
        self.processes.append(p)

    def _run_runtime(self) -> None:
        redirect_output(self.runtime.process_log_path(self.name, self.rank_in_replica))
        die_with_parent()
        logging.basicConfig(level=logging.INFO, format="%(asctime)s %(name)s %(levelname)s %(message)s")
        log.info("%s %s rank %d starting on %s", self.info.role, self.name, self.rank_in_replica, self.device)
        try:
            engine = self.build_engine()
            engine.setup()
            colocation = self.build_colocation_manager(engine)
            if colocation is not None:
                colocation.start()
            worker = self.build_worker(engine, colocation)
        except BaseException as e:  # report and exit: the parent's readiness wait fails fast
            log.exception("%s failed to start", self.name)
            try:
                self._error.put(repr(e))
            except Exception:
                pass
            raise
        if not self.is_master:
            engine.run_command_loop()
            return
        self._ready.set()
        try:
            worker.run()
        finally:
            try:
                engine.stop()
            except Exception:
                pass

    def wait_for_ready(self, timeout: float = 3600.0) -> None:
        if not self.is_master:
            return
        deadline = time.monotonic() + timeout
        while not self._ready.wait(timeout=0.5):
            if self.proc is not None and not self.proc.is_alive():
                err = None
                try:
                    err = self._error.get_nowait()
                except Exception:
                    pass
                raise RuntimeError(f"{self.info.role} {self.name} exited before ready: {err}")
            if time.monotonic() > deadline:
                raise TimeoutError(f"{self.info.role} {self.name} not ready within {timeout}s")
        self.runtime.mark_ready(self.name)
        log.info("%s %s ready", self.info.role, self.name)

    def health_info(self) -> dict[str, Any]:
        return {"name": self.name, "role": self.info.role, "rank": self.rank_in_replica,
                "alive": bool(self.proc is not None and self.proc.is_alive())}


__all__ = ["SpmdService", "current_rank", "require_ring"]
