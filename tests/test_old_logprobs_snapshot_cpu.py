"""``train_step`` takes the behaviour policy's log-probs before the first optimizer step.

Mirrors the reference's snapshot check (``tests/test_old_logprobs_snapshot.py``). With
``old_logprobs_source="train"`` every mini-batch must train against log-probs of the weights the rollout was
generated with: taking them inside each mini-batch would use weights already moved by the earlier
mini-batches, pin the ratio at 1 and switch the PPO clip / TIS off. ``train_step`` runs unbound on a stub, so
no model, GPU or process group is needed.
"""

from types import SimpleNamespace

import pytest
import torch

from meshy_b200.backend import trainer as T
from meshy_b200.backend.opd import StudentTopKTrainer


def _run(source: str, needs: bool = True, n_mini: int = 3):
    state = {"version": 0, "snapshots": [], "seen": []}

    def compute_old(samples, mini):
        state["snapshots"].append(state["version"])  # tag the snapshot with the weight version
        return [torch.tensor(float(state["version"]))]

    def run_mini(samples, mini, timer, old_lps=None):
        state["seen"].append(None if old_lps is None else float(old_lps[0]))
        state["version"] += 1  # this mini-batch's optimizer step
        return {"loss": 0.0}, torch.tensor(1.0)

    stub = SimpleNamespace(
        timer_enabled=False, needs_behaviour_logprobs=needs, batch_layout="padded", step=0,
        params=SimpleNamespace(enable_gae=False, old_logprobs_source=source),
        config=SimpleNamespace(warmup_steps=0, steps=10, lr_decay_ratio=0.0, lr_decay_type="linear",
                               lr_min_factor=0.0),
        optimizer=SimpleNamespace(lr=1e-6, base_lr=1e-6),
        compute_old_logprobs=compute_old, _run_mini_batch=run_mini,
    )
    plan = [SimpleNamespace(micros=[0]) for _ in range(n_mini)]
    mp = pytest.MonkeyPatch()
    mp.setattr(T, "plan_stats", lambda plan, layout: {})
    try:
        out = T.PPOTrainer.train_step(stub, [], plan=plan)
    finally:
        mp.undo()
    assert out["num_mini_batches"] == float(n_mini) and out["step"] == 1
    return state


def test_train_source_snapshots_every_mini_batch_before_any_step():
    s = _run("train")
    assert s["snapshots"] == [0, 0, 0]  # all taken at version 0
    assert s["seen"] == [0.0, 0.0, 0.0]  # later mini-batches still see the version-0 policy
    assert s["version"] == 3


def test_rollout_source_takes_no_snapshot():
    s = _run("rollout")
    assert s["snapshots"] == [] and s["seen"] == [None, None, None]


def test_trainer_without_a_ratio_skips_the_snapshot():
    s = _run("train", needs=False)
    assert s["snapshots"] == [] and s["seen"] == [None, None, None]


def test_distillation_trainer_opts_out():
    assert T.PPOTrainer.needs_behaviour_logprobs.fget(None) is True
    assert StudentTopKTrainer.needs_behaviour_logprobs.fget(None) is False
