"""Actor trainer service (reference ``meshy/service/training.py:31-191``).

Wiring only: ``from_info`` validates the ring membership of a colocated
trainer; the child builds a :class:`~meshy_b200.engine.trainer.TrainerEngine`
(one replica = ``n_gpus_per_replica`` DP ranks) and a
:class:`~meshy_b200.worker.trainer.TrainerWorker` that fetches rollout rows
from the column store, trains, publishes the next generation gate and hands
the card back through the ring with the new weights as ``payload_ref``.

``stream_minibatch`` makes the worker fetch ``mini_batch_size x dp`` rows per
pass and sync only after a full ``batch_size`` (the reference's streamed
mini-batch mode, ``meshy/service/training.py:177-180``).
"""

from __future__ import annotations

import os

from .checkpoint import run_resume_step
from .spmd import SpmdService, require_ring


class TrainingService(SpmdService):
    @classmethod
    def from_info(cls, info, topology, runtime, my_gpu=None):
        require_ring(info)
        return cls(info, topology, runtime, my_gpu)

    def _critic_cold_start(self) -> int:
        cfg = self.info.config
        if cfg.critic_cold_start_windows:
            return int(cfg.critic_cold_start_windows)
        return int(self.topology.cold_start_windows()) if self.topology is not None else 0

    def build_engine(self):
        from ..engine.trainer import TrainerEngine

        cfg = self.info.config
        eng = TrainerEngine(cfg.trainer_config, cfg.trainer_params, service_name=self.name, runtime=self.runtime,
                            checkpoint=cfg.checkpoint, weight_sync_mode=self.weight_sync_mode(),
                            weights_keep_latest_k=cfg.weights_keep_latest_k,
                            critic_cold_start_windows=self._critic_cold_start(), model_path=cfg.model_path,
                            **self.engine_kwargs())
        return eng

    def weight_sync_mode(self) -> str:
        """``auto`` becomes ``disk`` when the trainer's cards and the inference engines' cards are not all on
        one host: CUDA IPC handles only open on the node that exported them."""
        mode = self.info.config.weight_sync_mode
        if mode != "auto" or self.topology is None:
            return mode
        hosts = {g.host for g in self.info.replica_gpus}
        for svc in self.topology.inference_services():
            hosts |= {g.host for g in svc.replica_gpus}
        return "disk" if len(hosts) > 1 else mode

    def _chunk(self) -> int | None:
        cfg = self.info.config
        if not cfg.stream_minibatch:
            return None
        tp = cfg.trainer_params
        mini = getattr(tp, "mini_batch_size", None) if tp is not None else None
        if not mini:
            raise ValueError("stream_minibatch needs trainer_params.mini_batch_size")
        return int(mini) * self.world_size

    def build_worker(self, engine, colocation):
        from ..worker.trainer import TrainerWorker

        cfg = self.info.config
        resume = run_resume_step()
        engine.restore_counters(resume)
        worker = TrainerWorker(engine=engine, endpoints_ref=self.runtime_tq_ref(), partition_id=cfg.partition_id,
                               fields=cfg.tq_fields, batch_size=cfg.batch_size, chunk_size=self._chunk(),
                               poll_interval=cfg.tq_poll_interval, colocation=colocation,
                               gate_offset=self._critic_cold_start(), resume_step=resume)
        if os.environ.get("XRL_TENSORBOARD", "1") != "0" and self.is_master:
            from ..utils.metrics_adapter import MetricsWriter

            writer = MetricsWriter(self.runtime.tensorboard_path(self.name))
            worker.on_step = lambda res: writer.write(res.metrics, res.global_step)
        return worker


__all__ = ["TrainingService"]
