"""On-policy distillation services (reference ``meshy/service/opd.py:22-187``).

* :class:`OPDTrainingService` — the actor training service running the student Top-K engine;
* :class:`OPDTeacherService` — a frozen teacher replica appending Top-K columns to rollout rows.
"""

from __future__ import annotations

from .spmd import SpmdService, require_ring
from .training import TrainingService


class OPDTrainingService(TrainingService):
    def build_engine(self):
        from ..engine.opd import StudentTopKEngine

        cfg = self.info.config
        return StudentTopKEngine(cfg.trainer_config, cfg.trainer_params, service_name=self.name, runtime=self.runtime,
                                 checkpoint=cfg.checkpoint, weight_sync_mode=cfg.weight_sync_mode,
                                 weights_keep_latest_k=cfg.weights_keep_latest_k, critic_cold_start_windows=0,
                                 model_path=cfg.model_path, log_prob_min_clamp=cfg.log_prob_min_clamp,
                                 loss_max_clamp=cfg.loss_max_clamp, **self.engine_kwargs())


class OPDTeacherService(SpmdService):
    @classmethod
    def from_info(cls, info, topology, runtime, my_gpu=None):
        require_ring(info)
        return cls(info, topology, runtime, my_gpu)

    def build_engine(self):
        from ..engine.opd import OPDTeacherEngine

        return OPDTeacherEngine(self.info.config, **self.engine_kwargs())

    def build_worker(self, engine, colocation):
        from ..worker.opd import OPDTeacherWorker

        cfg = self.info.config
        return OPDTeacherWorker(engine=engine, endpoints_ref=self.runtime_tq_ref(), partition_id=cfg.partition_id,
                                batch_size=cfg.score_batch_size, poll_interval=cfg.tq_poll_interval,
                                colocation=colocation)


__all__ = ["OPDTeacherService", "OPDTrainingService"]
