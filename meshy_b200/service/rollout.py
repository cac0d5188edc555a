"""CPU rollout service (reference ``meshy/service/rollout.py:92-180``).

Started once, by global rank 0, after its ``wait_until`` groups are ready.
The child process runs a :class:`~meshy_b200.worker.rollout.RolloutWorker`
over an :class:`~meshy_b200.engine.rollout_client.EngineClient` that
round-robins the inference replicas' HTTP endpoints (replica-level data
parallelism of inference), writes rollout groups to the column store and
follows the trainer's generation gates.
"""

from __future__ import annotations

import logging
import multiprocessing
import os
import time

from .base import Service, die_with_parent, redirect_output

log = logging.getLogger(__name__)


class RolloutService(Service):
    def __init__(self, info, topology, runtime, my_gpu=None):
        super().__init__(info, topology, runtime)
        self.processes: list = []
        self._ready = None

    @classmethod
    def from_info(cls, info, topology, runtime, my_gpu=None):
        return cls(info, topology, runtime, my_gpu)

    def _train_batch_size(self) -> int:
        ts = self.topology.training_services() if self.topology is not None else []
        if ts:
            return int(ts[0].config.batch_size)
        return int(getattr(self.info.config, "train_batch_size", 0) or 0)

    def build_worker(self):
        from ..engine.rollout_client import EngineClient
        from ..worker.rollout import RolloutWorker
        from .checkpoint import run_resume_step

        cfg = self.info.config
        endpoints = self.topology.inference_endpoints()
        client = EngineClient(endpoints, cfg.sampling_params)
        client.model_path = cfg.model_path
        traj = cfg.trajectory_log or self.runtime.trajectory_path()
        return RolloutWorker(
            engine=client, endpoints_ref=cfg.tq_endpoints_file or os.environ.get("XRL_TQ_ENDPOINTS"),
            model_path=cfg.model_path, dataset=cfg.dataset, dataset_kwargs=cfg.dataset_kwargs,
            partition_id=cfg.partition_id, group_size=cfg.group_size, train_batch_size=self._train_batch_size(),
            sampling_params=cfg.sampling_params, reward=cfg.reward, reward_shaping=cfg.reward_shaping,
            reward_shaping_kwargs=cfg.reward_shaping_kwargs, advantage=cfg.advantage,
            advantage_kwargs=cfg.advantage_kwargs, filter_zero_std_groups=cfg.filter_zero_std_groups,
            publish_positive_lm_weights=cfg.publish_positive_lm_weights, oversample_factor=cfg.oversample_factor,
            num_epochs=cfg.num_epochs, pacing_window=cfg.pacing_window,
            max_running_requests=cfg.async_max_running_request, poll_interval=cfg.poll_interval,
            trajectory_log=traj, verbose_trajectory_log=cfg.verbose_trajectory_log,
            external_advantage=cfg.external_advantage, checkpoint=cfg.checkpoint, resume_step=run_resume_step(),
            state_dir=self.runtime.state_dir, service_name=self.name)

    def ignite(self) -> None:
        ctx = multiprocessing.get_context("spawn")
        self._ready = ctx.Event()
        p = ctx.Process(target=self._run, name=self.name)
        p.start()
        self.proc = p
        self.processes.append(p)

    def _run(self) -> None:
        redirect_output(self.runtime.process_log_path(self.name, 0))
        die_with_parent()
        logging.basicConfig(level=logging.INFO, format="%(asctime)s %(name)s %(levelname)s %(message)s")
        worker = self.build_worker()
        self._ready.set()
        worker.run()

    def wait_for_ready(self, timeout: float = 600.0) -> None:
        deadline = time.monotonic() + timeout
        while not self._ready.wait(timeout=0.5):
            if not self.proc.is_alive():
                raise RuntimeError(f"rollout {self.name} exited before ready")
            if time.monotonic() > deadline:
                raise TimeoutError(f"rollout {self.name} not ready within {timeout}s")
        self.runtime.mark_ready(self.name)


__all__ = ["RolloutService"]
