"""SPMD replica engine: one process per card, rank 0 drives, the rest follow.

Each replica gets its own process groups: NCCL (CUDA) or gloo (CPU) for
compute and a gloo group for control.  Rank 0's worker calls
:meth:`SpmdEngine.submit_command`; the command is broadcast to every rank
(``broadcast_object_list`` on the control group) and executed collectively
as ``cmd_<name>(payload)``; ranks > 0 sit in :meth:`run_command_loop`.
Reference: ``meshy/engine/spmd.py:91-261``.
"""

from __future__ import annotations

import logging
import os
import threading
from datetime import timedelta
from typing import Any

import torch
import torch.distributed as dist

log = logging.getLogger(__name__)
DEFAULT_TIMEOUT_S = float(os.environ.get("XRL_SPMD_TIMEOUT_S", str(8 * 3600)))
_ELASTIC_VARS = ("TORCHELASTIC_RUN_ID", "TORCHELASTIC_RESTART_COUNT", "TORCHELASTIC_MAX_RESTARTS",
                 "TORCHELASTIC_USE_AGENT_STORE", "GROUP_RANK", "ROLE_RANK", "ROLE_WORLD_SIZE", "LOCAL_WORLD_SIZE",
                 "GROUP_WORLD_SIZE", "ROLE_NAME")


class SpmdEngine:
    def __init__(self, *, rank: int, world_size: int, master_addr: str = "127.0.0.1", master_port: int = 29500,
                 device: str | torch.device = "cpu", timeout_s: float | None = None):
        self.rank = rank
        self.world_size = world_size
        self.master_addr = master_addr
        self.master_port = master_port
        self.device = torch.device(device)
        self.timeout = timedelta(seconds=timeout_s or DEFAULT_TIMEOUT_S)
        self.control_group = None
        self.compute_group = None
        self._running = False
        # rank 0 submits from the worker thread and from the colocation manager's callbacks; one
        # lock keeps the broadcast order (and so the collective order) identical on every rank
        self._cmd_lock = threading.Lock()

    def init_process_group(self) -> None:
        for v in _ELASTIC_VARS:
            os.environ.pop(v, None)
        os.environ["MASTER_ADDR"] = self.master_addr
        os.environ["MASTER_PORT"] = str(self.master_port)
        if self.device.type == "cuda":
            # collectives that stage through the current device (all_gather_object and friends) must
            # see the device the process group was bound to
            torch.cuda.set_device(self.device)
        if not dist.is_initialized():
            backend = "nccl" if self.device.type == "cuda" else "gloo"
            kw = {"device_id": self.device} if backend == "nccl" else {}
            dist.init_process_group(backend, rank=self.rank, world_size=self.world_size, timeout=self.timeout, **kw)
        self.compute_group = dist.group.WORLD
        self.control_group = dist.new_group(backend="gloo", timeout=self.timeout)

    # ------------------------------------------------------------------ commands
    def submit_command(self, name: str, payload: Any = None) -> Any:
        if self.rank != 0:
            raise RuntimeError("only rank 0 submits commands")
        with self._cmd_lock:
            return self._broadcast_and_run([name, payload])

    def _broadcast_and_run(self, obj) -> Any:
        if self.world_size > 1:
            box = [obj]
            dist.broadcast_object_list(box, src=0, group=self.control_group)
            obj = box[0]
        name, payload = obj
        if name == "__stop__":
            self._running = False
            return None
        return getattr(self, f"cmd_{name}")(payload)

    def run_command_loop(self) -> None:
        self._running = True
        while self._running:
            self._broadcast_and_run([None, None])

    def setup(self) -> None:
        if self.world_size > 1 and not dist.is_initialized():
            self.init_process_group()

    def stop(self) -> None:
        if self.rank == 0 and self.world_size > 1:
            with self._cmd_lock:
                self._broadcast_and_run(["__stop__", None])

    def barrier(self) -> None:
        if self.world_size > 1:
            dist.barrier(group=self.control_group)

    def broadcast_object(self, obj=None):
        if self.world_size == 1:
            return obj
        box = [obj]
        dist.broadcast_object_list(box, src=0, group=self.control_group)
        return box[0]


__all__ = ["SpmdEngine"]
