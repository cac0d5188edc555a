"""Critic service (reference ``meshy/service/critic.py:28-217``): an SPMD replica running the
:class:`~meshy_b200.engine.critic.CriticSpmdEngine` and :class:`~meshy_b200.worker.critic.CriticWorker`."""

from __future__ import annotations

import os

from .checkpoint import run_resume_step
from .spmd import SpmdService, require_ring


class CriticService(SpmdService):
    @classmethod
    def from_info(cls, info, topology, runtime, my_gpu=None):
        require_ring(info)
        return cls(info, topology, runtime, my_gpu)

    def build_engine(self):
        from ..engine.critic import CriticSpmdEngine

        return CriticSpmdEngine(self.info.config, service_name=self.name, runtime=self.runtime,
                                **self.engine_kwargs())

    def _actor_weights(self):
        trainers = self.topology.training_services() if self.topology is not None else []
        if not trainers:
            return None
        name = trainers[0].name
        rt = self.runtime

        def path(version: int):
            p = rt.checkpoint_path(name, version)
            return p if os.path.isdir(p) else None

        return path

    def build_worker(self, engine, colocation):
        from ..worker.critic import CriticWorker

        cfg = self.info.config
        resume = run_resume_step()
        if resume > 0:
            engine.restore_state(resume)
        worker = CriticWorker(engine=engine, endpoints_ref=self.runtime_tq_ref(), partition_id=cfg.partition_id,
                              batch_size=cfg.score_batch_size, output_field=cfg.output_fields[0],
                              cold_start_windows=cfg.cold_start_windows, poll_interval=cfg.tq_poll_interval,
                              colocation=colocation, actor_weights=self._actor_weights(), resume_windows=resume)
        if self.is_master and os.environ.get("XRL_TENSORBOARD", "1") != "0":
            from ..utils.metrics_adapter import MetricsWriter

            writer = MetricsWriter(self.runtime.tensorboard_path(self.name))
            worker.on_window = lambda res, step: writer.write(res.get("metrics", {}), step)
        return worker


__all__ = ["CriticService"]
