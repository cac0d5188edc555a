"""Actor training engine (the reference's ``TitanEngine``, ``meshy/engine/titan.py:126-560``).

``step(samples, sync)`` on rank 0 broadcasts the window, every rank plans the
global batch identically and trains its DP slice (:class:`PPOTrainer`), then
on ``sync`` the engine bumps the weight version, publishes weights (device IPC
handle for same-node engines, or an HF safetensors export), takes the global
checkpoint when due and rotates old exports while protecting versions a
retained checkpoint still points at.  Offload/restore implement the
colocation hand-off.
"""

from __future__ import annotations

import logging
import os
import shutil
import time
from dataclasses import dataclass, field
from typing import Any

import torch

from ..backend.trainer import PPOTrainer
from ..config import GlobalCheckpointConfig, TrainerConfig, TrainerParamsConfig
from .spmd import SpmdEngine

log = logging.getLogger(__name__)


@dataclass
class StepResult:
    metrics: dict = field(default_factory=dict)
    weight_version: int = 0
    weights_ref: str | None = None
    global_step: int = 0


class TrainerEngine(SpmdEngine):
    def __init__(self, trainer_config: TrainerConfig, trainer_params: TrainerParamsConfig | None, *, service_name: str,
                 runtime=None, checkpoint: GlobalCheckpointConfig | None = None, weight_sync_mode: str = "auto",
                 weights_keep_latest_k: int = 5, critic_cold_start_windows: int = 0, model_path: str | None = None,
                 **kw):
        super().__init__(**kw)
        self.tc, self.tp = trainer_config, trainer_params
        self.service_name = service_name
        self.runtime = runtime
        self.checkpoint = GlobalCheckpointConfig.coerce(checkpoint)
        self.weight_sync_mode = weight_sync_mode
        self.weights_keep_latest_k = weights_keep_latest_k
        self.cold = int(critic_cold_start_windows)
        self.model_path = model_path
        self.trainer: PPOTrainer | None = None
        self.version = 0
        self.step_index = 0

    def setup(self) -> None:
        if self.world_size > 1 and not torch.distributed.is_initialized():
            self.init_process_group()
        groups = self.parallel_groups()
        self.trainer = PPOTrainer(self.tc, self.tp, device=self.device, **groups)
        if self.model_path and os.path.isdir(self.model_path):
            from ..models.hf import load_hf_checkpoint

            self.trainer.flat.load_state_dict(load_hf_checkpoint(self.trainer.model_args, self.model_path))

    def parallel_groups(self) -> dict:
        """DP / CP / loss groups of this replica from the trainer config's parallel degrees."""
        if self.world_size == 1:
            return {"dp_group": None}
        from ..parallel.mesh import build_parallel_dims

        tc = self.tc
        cp = max(1, int(getattr(tc, "cp_degree", 1)))
        ep = max(1, int(getattr(tc, "ep_degree", 1)))
        if self.shard_parameters():
            rep = max(1, int(getattr(tc, "dp_replicate_degree", 1)))
            pd = build_parallel_dims(self.world_size, self.rank, dp_replicate=rep, dp_shard=-1, cp=cp,
                                     tp=max(1, int(getattr(tc, "tp_degree", 1))))
            self.parallel_dims = pd
            return {"dp_group": pd.batch_group, "cp_group": pd.cp_group, "loss_group": pd.loss_group,
                    "tp_group": pd.tp_group, "fsdp_group": pd.shard_group, "replicate_group": pd.replicate_group}
        if cp == 1 and int(getattr(tc, "tp_degree", 1)) <= 1:
            out = {"dp_group": self.compute_group}
            if ep > 1:
                if ep != self.world_size:
                    raise ValueError("ep_degree must equal the replica's DP size (experts split over the DP ranks)")
                out["ep_group"] = self.compute_group
            return out
        pd = build_parallel_dims(self.world_size, self.rank, dp_replicate=-1, dp_shard=1, cp=cp,
                                 tp=max(1, int(getattr(tc, "tp_degree", 1))))
        self.parallel_dims = pd
        return {"dp_group": pd.batch_group, "cp_group": pd.cp_group, "loss_group": pd.loss_group,
                "tp_group": pd.tp_group}

    def shard_parameters(self) -> bool:
        """Whether this replica shards its parameters (``shard_params``; "auto": the replicated state -- bf16
        weights, fp32 gradients, and the fp32 master and moments split over the ranks -- above 40 % of HBM)."""
        mode = getattr(self.tc, "shard_params", "auto")
        if mode != "auto" or self.world_size == 1:
            return mode == "on" and self.world_size > 1
        if self.device.type != "cuda" or int(getattr(self.tc, "ep_degree", 1)) > 1 \
                or int(getattr(self.tc, "tp_degree", 1)) > 1:
            return False
        from ..models import get_model_args

        n = get_model_args(self.tc.model_name, self.tc.model_flavor).num_params()
        need = n * (2 + 4 + 12 / self.world_size)
        return need > 0.4 * torch.cuda.get_device_properties(self.device).total_memory

    @property
    def global_step(self) -> int:
        return self.step_index + self.cold

    # ------------------------------------------------------------------ public (rank 0)
    def step(self, samples: list[dict], sync: bool = True) -> StepResult:
        return self.submit_command("step", {"samples": samples, "sync": sync})

    def offload(self) -> None:
        self.submit_command("offload", None)

    def restore(self) -> None:
        self.submit_command("restore", None)

    # ------------------------------------------------------------------ collective commands
    def cmd_step(self, payload) -> StepResult:
        samples, sync = payload["samples"], payload["sync"]
        t = self.trainer
        plan = t.plan_batch(samples, t.dp_size)
        local = plan.local_samples(samples, t.dp_rank)  # CP / TP ranks of one DP index get the same share
        t0 = time.perf_counter()
        metrics = t.train_step(local, plan=plan.per_rank[t.dp_rank], step_schedule=sync)
        metrics["time/train/step"] = time.perf_counter() - t0
        res = StepResult(metrics=metrics)
        if sync:
            self.step_index += 1
            self.version += 1
            res.weight_version = self.version
            res.global_step = self.global_step
            res.weights_ref = self.publish_weights()
            if self.checkpoint.due(self.global_step):
                self.save_global_checkpoint(self.global_step)
        return res

    # colocation ring callbacks (rank 0, manager thread): every rank changes residency together
    def on_colocate_acquire(self, grant) -> None:
        self.restore()

    def on_colocate_release(self, target: str) -> None:
        self.offload()

    def cmd_offload(self, payload) -> None:
        self.trainer.offload_to_cpu()

    def cmd_restore(self, payload) -> None:
        self.trainer.restore_to_gpu()

    # ------------------------------------------------------------------ weights
    def publish_weights(self) -> str | None:
        """Make this step's weights available to the inference engines; returns the reference that travels
        through the colocation ring as ``payload_ref`` (rank 0; other ranks return ``None``).

        Device path (``weight_sync_mode`` ``device``, or ``auto`` when every trainer rank and the engines
        share one node): every rank casts its fp32 master weights into a bf16 snapshot in the engines'
        flat layout (:class:`~meshy_b200.rollout.weight_sync.DevicePublisher`) and exports a CUDA IPC handle
        of it; rank 0 gathers the handles keyed by GPU UUID into one ``ipc-set:`` reference, and each
        engine copies the snapshot of the trainer rank on its own GPU. No disk, no gather of weights.
        Disk path: an HF safetensors export (also the checkpoint format), as the reference does for
        every sync (``meshy/engine/titan.py:80-123``)."""
        mode = self.weight_sync_mode
        if mode in ("auto", "device") and self.device.type == "cuda" and self._replicated_weights() and (
                mode == "device" or self._single_node()):
            from ..rollout.weight_sync import DevicePublisher, encode_handle_set

            if getattr(self, "_publisher", None) is None:
                self._publisher = DevicePublisher(self.trainer.flat, self.device)
            entry = self._publisher.publish(self.version)
            entries = self.gather_objects(entry)
            return encode_handle_set(entries) if self.rank == 0 else None
        if self.runtime is None:
            return None
        path = self.runtime.checkpoint_path(self.service_name, self.version)
        self._export_hf(path)
        if self.rank == 0:
            self.prune_weights()
        self.barrier()
        return path

    def _export_hf(self, path: str) -> None:
        """HF safetensors export, written by rank 0. With sharded parameters every rank takes part in gathering
        the full weights first (a collective), then rank 0 writes them."""
        if getattr(self.trainer.flat, "sharded", False):
            from ..models.hf import save_hf_checkpoint

            sd = self.trainer.flat.state_dict(source="compute")
            if self.rank == 0:
                save_hf_checkpoint(self.trainer.model_args, sd, path)
        elif self.rank == 0:
            self.trainer.export_hf(path)

    def _replicated_weights(self) -> bool:
        """Whether every rank holds the whole model (DP / CP): expert- or tensor-parallel ranks hold parts."""
        t = self.trainer
        sharded = [g for g in (t.ep_group, t.tp_group) if g is not None and torch.distributed.is_initialized()
                   and torch.distributed.get_world_size(g) > 1]
        return not sharded

    def _single_node(self) -> bool:
        """Whether every rank of this replica runs on this host (the IPC handles only open there)."""
        if self.world_size == 1:
            return True
        if getattr(self, "_hosts_same", None) is None:
            import socket

            hosts = self.gather_objects(socket.gethostname())
            same = None
            if self.rank == 0:
                same = len(set(hosts)) == 1
            self._hosts_same = bool(self.broadcast_object(same))
        return self._hosts_same

    def gather_objects(self, obj) -> list | None:
        """Every rank's ``obj`` on rank 0 (``None`` elsewhere), over the gloo control group."""
        if self.world_size == 1 or not torch.distributed.is_initialized():
            return [obj]
        out = [None] * self.world_size if self.rank == 0 else None
        torch.distributed.gather_object(obj, out, dst=0, group=self.control_group)
        return out

    def prune_weights(self) -> list[int]:
        if self.runtime is None or self.weights_keep_latest_k <= 0:
            return []
        wdir = self.runtime.weights_dir(self.service_name)
        try:
            versions = sorted(int(d[1:]) for d in os.listdir(wdir) if d.startswith("v") and d[1:].isdigit())
        except FileNotFoundError:
            return []
        protected = set()
        store = self.runtime.state_store()
        for step in store.complete_steps(self.service_name):
            v = store.payload(self.service_name, step).get("weight_version")
            if v is not None:
                protected.add(int(v))
        stale = [v for v in versions[:-self.weights_keep_latest_k] if v not in protected]
        for v in stale:
            shutil.rmtree(os.path.join(wdir, f"v{v}"), ignore_errors=True)
        return stale

    # ------------------------------------------------------------------ checkpoints
    def save_global_checkpoint(self, step: int) -> None:
        store = self.runtime.state_store()
        # a resumed run boots its engines from the HF export of the checkpointed weight version; with
        # device weight sync no per-step export exists, so the checkpoint writes that one
        path = self.runtime.checkpoint_path(self.service_name, self.version)
        missing = self.broadcast_object(not os.path.isdir(path) if self.rank == 0 else None)
        if missing:
            self._export_hf(path)
            if self.rank == 0:
                self.prune_weights()
        self.trainer.save_checkpoint(store.shard_dir(self.service_name, step), step)
        if self.rank == 0:
            store.write_meta(self.service_name, step, {"step_index": self.step_index, "weight_version": self.version,
                                                       "trainer_step": self.trainer.step})
            store.mark_complete(self.service_name, step)
            store.prune(self.service_name, self.checkpoint.keep_latest_k)
        self.barrier()

    def restore_counters(self, resume_step: int) -> None:
        if resume_step <= 0 or self.runtime is None:
            return
        store = self.runtime.state_store()
        if not store.is_complete(self.service_name, resume_step):
            if resume_step <= self.cold:  # trainer idle during the critic cold start
                self.step_index = 0
                return
            raise FileNotFoundError(f"no trainer shard at global step {resume_step}")
        p = store.payload(self.service_name, resume_step)
        self.trainer.load_checkpoint(store.shard_dir(self.service_name, resume_step))
        self.step_index = int(p["step_index"])
        self.version = int(p["weight_version"])


__all__ = ["StepResult", "TrainerEngine"]
