"""Generation gates: the trainer's "rollout may start step N" pulses.

One rolling two-column partition (``gate_step``, ``weight_version``); the
rollout fetches one row per step as task ``gen_gate`` and clears it, so the
stream stays O(1) (reference ``meshy/transferqueue/control.py:49-156``).
"""

from __future__ import annotations

import logging
import time

import torch

from .client import Columns

log = logging.getLogger(__name__)

GEN_GATE_PARTITION = "gen_gate"
GEN_GATE_STEP_FIELD = "gate_step"
GEN_GATE_VERSION_FIELD = "weight_version"
GEN_GATE_FIELDS = [GEN_GATE_STEP_FIELD, GEN_GATE_VERSION_FIELD]
GEN_GATE_TASK = "gen_gate"


def make_gen_gate(step: int, weight_version: int = -1) -> Columns:
    return Columns({GEN_GATE_STEP_FIELD: [torch.tensor([int(step)])],
                    GEN_GATE_VERSION_FIELD: [torch.tensor([int(weight_version)])]})


def emit_gen_gate(client, step: int, weight_version: int = -1):
    return client.put(data=make_gen_gate(step, weight_version), partition_id=GEN_GATE_PARTITION)


def read_gen_gate(client, step: int) -> int | None:
    meta = client.get_meta(data_fields=GEN_GATE_FIELDS, batch_size=1, partition_id=GEN_GATE_PARTITION, mode="fetch",
                           task_name=GEN_GATE_TASK)
    if meta.size < 1:
        return None
    data = client.get_data(meta)
    gate_step = int(data[GEN_GATE_STEP_FIELD][0].reshape(-1)[0])
    version = int(data[GEN_GATE_VERSION_FIELD][0].reshape(-1)[0])
    client.clear_samples(meta)
    if gate_step != int(step):
        log.warning("gen_gate stream out of order: expected step %s, got %s (weight_version=%s)", step, gate_step,
                    version)
    return version


def wait_gen_gate(client, step: int, *, interval: float = 0.5, timeout: float | None = None) -> int:
    start = time.monotonic()
    while True:
        v = read_gen_gate(client, step)
        if v is not None:
            return v
        if timeout is not None and time.monotonic() - start > timeout:
            raise TimeoutError(f"timed out after {timeout}s waiting for gen gate step {step}")
        time.sleep(interval)


__all__ = ["GEN_GATE_FIELDS", "GEN_GATE_PARTITION", "GEN_GATE_STEP_FIELD", "GEN_GATE_TASK", "GEN_GATE_VERSION_FIELD",
           "emit_gen_gate", "make_gen_gate", "read_gen_gate", "wait_gen_gate"]
