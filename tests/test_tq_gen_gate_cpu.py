"""Generation-gate stream over the in-process native column store (CPU only).

Mirrors the reference's gate checks (``tests/test_tq_gen_gate.py``): the gate is the signal that paces the
whole run, so its semantics are pinned against the real store, not a fake.

* a gate not yet raised reads as ``None`` (never raises, never blocks);
* a raised gate is read exactly once and carries its weight version;
* gates come back in emission order;
* every read clears its row, so a long run keeps the stream O(1);
* ``wait_gen_gate`` gives up with ``TimeoutError``;
* the trainer worker's genesis gate is 0 on a fresh run, follows the critic's cold-start gates when there
  are some, and re-establishes the stream at the resume step after a restart.
"""

from types import SimpleNamespace

import pytest

from meshy_b200.tq import control
from meshy_b200.tq.client import LocalClient


@pytest.fixture()
def client():
    return LocalClient()


def test_unraised_gate_reads_as_none(client):
    assert control.read_gen_gate(client, 0) is None


def test_gate_roundtrip_and_single_consumption(client):
    control.emit_gen_gate(client, step=0, weight_version=7)
    assert control.read_gen_gate(client, 0) == 7
    assert control.read_gen_gate(client, 1) is None


def test_gates_arrive_in_emission_order(client):
    for step in (1, 2, 3):
        control.emit_gen_gate(client, step=step, weight_version=step)
    assert [control.read_gen_gate(client, s) for s in (1, 2, 3, 4)] == [1, 2, 3, None]


def test_gate_stream_stays_bounded(client):
    for step in range(200):
        control.emit_gen_gate(client, step=step, weight_version=step)
        assert control.read_gen_gate(client, step) == step
    assert client.store.num_rows(control.GEN_GATE_PARTITION) == 0


def test_wait_gen_gate_times_out_cleanly(client):
    with pytest.raises(TimeoutError):
        control.wait_gen_gate(client, step=999, interval=0.05, timeout=0.3)
    control.emit_gen_gate(client, step=5, weight_version=3)
    assert control.wait_gen_gate(client, step=5, interval=0.01, timeout=1.0) == 3


def _genesis(resume_step, cold_start):
    from meshy_b200.worker.trainer import TrainerWorker

    w = TrainerWorker(engine=SimpleNamespace(version=resume_step), endpoints_ref=None, partition_id="data.train",
                      fields=["tokens"], batch_size=8, gate_offset=cold_start, resume_step=resume_step,
                      client_factory=LocalClient)
    cols = w.startup_tq_outputs()["gen_gate"]
    return int(cols[control.GEN_GATE_STEP_FIELD][0].reshape(-1)[0])


def test_genesis_gate_numbering():
    assert _genesis(resume_step=0, cold_start=0) == 0  # fresh run
    assert _genesis(resume_step=0, cold_start=20) == 20  # after the critic's cold-start gates 0..19
    assert _genesis(resume_step=35, cold_start=20) == 35  # a resumed run picks the stream up where it stopped
