"""Actor trainer role loop (reference ``meshy/worker/titan.py:14-150``).

Consumes ``batch_size`` rows of the trainer columns (task ``trainer``), asks
the colocation ring for the card, trains, releases the card with the new
weights' reference as ``payload_ref`` (the inference side loads them on
acquire), and raises the next generation gate.  Gate numbering starts above
the critic's cold start and is re-published at the resume step.  With
``stream_minibatch`` the trainer consumes mini-batch chunks and only syncs
(version, gate, LR step) once per ``batch_size``.
"""

from __future__ import annotations

import logging

import torch

from ..tq.client import Columns
from ..tq.control import GEN_GATE_FIELDS, GEN_GATE_PARTITION, make_gen_gate
from .tq import TQInput, TQOutput, TQWorker

log = logging.getLogger(__name__)


class TrainerWorker(TQWorker):
    def __init__(self, *, engine, endpoints_ref: str | None, partition_id: str, fields, batch_size: int,
                 chunk_size: int | None = None, poll_interval: float = 0.5, colocation=None,
                 gate_offset: int = 0, resume_step: int = 0, client_factory=None, on_step=None):
        super().__init__()
        self.engine = engine
        self.colocation = colocation
        self.batch_size = int(batch_size)
        self.chunk = int(chunk_size or batch_size)
        if self.batch_size % self.chunk:
            raise ValueError("batch_size must be a multiple of the streamed mini-batch chunk")
        self.consumed_in_window = 0
        self.gate_offset = int(gate_offset)
        self.resume_step = int(resume_step)
        self.on_step = on_step
        self.history: list[dict] = []
        self.configure_tq(endpoints_ref=endpoints_ref,
                          input=TQInput(partition_id, tuple(fields), self.chunk, "trainer", True),
                          outputs={"gen_gate": TQOutput(tuple(GEN_GATE_FIELDS), True, GEN_GATE_PARTITION)},
                          poll_interval=poll_interval, client_factory=client_factory)

    def startup_tq_outputs(self) -> dict[str, Columns]:
        """Genesis gate: step ``max(resume_step, gate_offset)`` releases the first window."""
        step = max(self.resume_step, self.gate_offset)
        return {"gen_gate": make_gen_gate(step, self.engine.version)}

    def process_tq_batch(self, samples: list[dict]) -> dict[str, Columns]:
        self.consumed_in_window += len(samples)
        sync = self.consumed_in_window >= self.batch_size
        req = None
        if self.colocation is not None:
            req = self.colocation.request_gpu()
            self.colocation.wait_for_grant(req)
        res = self.engine.step(samples, sync=sync)
        self.history.append(res.metrics)
        if self.on_step is not None:
            self.on_step(res)
        out: dict[str, Columns] = {}
        if sync:
            self.consumed_in_window = 0
            out["gen_gate"] = make_gen_gate(res.global_step, res.weight_version)
        if self.colocation is not None and sync:
            self.colocation.release(transition="trained", payload_ref=res.weights_ref)
        return out


__all__ = ["TrainerWorker"]
