"""Teacher role loop (reference ``meshy/worker/opd.py:17-87``): fetch rollout rows (task ``teacher``),
append the Top-K columns in place, never clear (the student trainer clears after training).
The student trainer's AND-filter fetch over ``OPD_TRAINER_FIELDS`` waits for those columns."""

from __future__ import annotations

import logging
from typing import Any, Mapping

from ..config import DEFAULT_DATA_PARTITION, OPD_TEACHER_FIELDS
from ..tq.client import Columns
from .tq import TQInput, TQOutput, TQWorker

log = logging.getLogger(__name__)
TEACHER_INPUT_FIELDS = ("tokens", "mask_assistant")


class OPDTeacherWorker(TQWorker):
    def __init__(self, *, engine, endpoints_ref: str | None, partition_id: str = DEFAULT_DATA_PARTITION,
                 batch_size: int, poll_interval: float = 0.5, colocation=None, client_factory=None):
        super().__init__()
        self.engine = engine
        self.colocation = colocation
        self.scored = 0
        self.configure_tq(endpoints_ref=endpoints_ref,
                          input=TQInput(partition_id, TEACHER_INPUT_FIELDS, batch_size, "teacher", False),
                          outputs={"topk": TQOutput(tuple(OPD_TEACHER_FIELDS), False, partition_id)},
                          poll_interval=poll_interval, client_factory=client_factory)

    def process_tq_batch(self, samples: list[Any]) -> Mapping[str, Any]:
        req = None
        if self.colocation is not None:
            req = self.colocation.request_gpu()
            self.colocation.wait_for_grant(req)
        try:
            res = self.engine.score(samples)
        finally:
            if req is not None:
                self.colocation.release(transition="teacher-scored")
        if res is None or len(res) != len(samples):
            raise RuntimeError("teacher returned the wrong number of rows")
        self.scored += len(samples)
        ids, lps = zip(*res)
        return {"topk": Columns({OPD_TEACHER_FIELDS[0]: list(ids), OPD_TEACHER_FIELDS[1]: list(lps)})}


__all__ = ["OPDTeacherWorker"]
