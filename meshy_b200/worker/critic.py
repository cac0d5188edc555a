"""Critic role loop (reference ``meshy/worker/critic.py:49-249``).

Consumes ``score_batch_size`` rollout rows (task ``critic``) that carry
``tokens``, ``mask_assistant``, ``reward`` and ``weight_version``.

* Cold start (the first ``cold_start_windows`` windows, or forever with a
  negative count): the critic only trains; nothing downstream reads these rows,
  so the critic clears them itself and raises the generation gate that paces
  the rollout while the actor is frozen.
* Warm: the critic publishes its output column (``values`` or ``advantage``)
  into the same rows and leaves them for the trainer, whose AND-filter fetch
  waits for that column; the trainer clears them.

Around each window it holds the colocation ring (when it is in one) and
releases with the actor weights the rows were generated against as
``payload_ref``, so the inference side reloads the right version.
"""

from __future__ import annotations

import logging
from typing import Any, Callable, Mapping

from ..config import CRITIC_INPUT_FIELDS, DEFAULT_DATA_PARTITION
from ..tq.client import Columns
from ..tq.control import GEN_GATE_FIELDS, GEN_GATE_PARTITION, make_gen_gate
from .tq import TQInput, TQOutput, TQWorker

log = logging.getLogger(__name__)


class CriticWorker(TQWorker):
    def __init__(self, *, engine, endpoints_ref: str | None, partition_id: str = DEFAULT_DATA_PARTITION,
                 batch_size: int, output_field: str = "values", cold_start_windows: int = 0,
                 poll_interval: float = 0.5, colocation=None, actor_weights: Callable[[int], str | None] | None = None,
                 resume_windows: int = 0, client_factory=None, on_window=None):
        super().__init__()
        self.engine = engine
        self.colocation = colocation
        self.output_field = output_field
        self.cold_start_windows = int(cold_start_windows)
        self.windows = int(resume_windows)
        self.gates_raised = int(resume_windows) if self.in_cold_start else 0
        self.actor_weights = actor_weights
        self.on_window = on_window
        self.configure_tq(endpoints_ref=endpoints_ref,
                          input=TQInput(partition_id, tuple(CRITIC_INPUT_FIELDS), batch_size, "critic", False),
                          outputs={output_field: TQOutput((output_field,), False, partition_id),
                                   "gate": TQOutput(tuple(GEN_GATE_FIELDS), True, GEN_GATE_PARTITION)},
                          poll_interval=poll_interval, client_factory=client_factory)

    @property
    def in_cold_start(self) -> bool:
        return self.cold_start_windows < 0 or self.windows < self.cold_start_windows

    def should_clear_batch(self) -> bool:
        # cold-start rows are read by nobody else; warm rows are cleared by the trainer
        return self._cleared_by_me

    def startup_tq_outputs(self) -> Mapping[str, Any]:
        if self.in_cold_start or self.cold_start_windows == 0:
            # genesis gate of the cold start (the trainer publishes it when there is none)
            return {"gate": make_gen_gate(self.gates_raised, 0)} if self.cold_start_windows else {}
        return {}

    def process_tq_batch(self, samples: list[Any]) -> Mapping[str, Any]:
        cold = self.in_cold_start
        self._cleared_by_me = cold
        self.windows += 1
        req = None
        if self.colocation is not None:
            req = self.colocation.request_gpu()
            self.colocation.wait_for_grant(req)
        try:
            result = self.engine.score_and_train(samples, publish=not cold, global_step=self.windows)
        finally:
            if req is not None:
                self.colocation.release(transition="critic-window-complete", payload_ref=self._actor_weights(samples))
        if result is None:
            raise RuntimeError("critic engine returned no result on its driving rank")
        log.info("critic %s %d: value_loss=%.4f rows=%d | %s", "cold start" if cold else "window", self.windows,
                 float(result.get("value_loss", float("nan"))), int(result.get("rows", 0)),
                 result.get("diagnostics"))
        if self.on_window is not None:
            self.on_window(result, self.windows)
        if cold:
            self.gates_raised += 1
            return {"gate": make_gen_gate(self.gates_raised, int(getattr(self.engine, "weight_version", 0)))}
        scored = result[self.output_field]
        if len(scored) != len(samples):
            raise ValueError(f"critic produced {len(scored)} {self.output_field} rows for {len(samples)} inputs")
        import torch

        return {self.output_field: Columns({self.output_field: [torch.tensor(x, dtype=torch.float32)
                                                                for x in scored]})}

    _cleared_by_me = False

    def _actor_weights(self, samples) -> str | None:
        if self.actor_weights is None:
            return None
        import torch

        v = max(int(torch.as_tensor(s["weight_version"]).reshape(-1)[0]) for s in samples)
        return self.actor_weights(v)

    def health_info(self) -> dict[str, Any]:
        info = super().health_info()
        info["critic"] = {"windows": self.windows, "cold_start_windows": self.cold_start_windows,
                          "in_cold_start": self.in_cold_start, "gates_raised": self.gates_raised}
        return info


__all__ = ["CriticWorker"]
