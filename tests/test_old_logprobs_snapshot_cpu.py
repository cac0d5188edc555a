"""The PPO ratio's denominator is the policy that generated the batch (CPU, real trainer).

With ``old_logprobs_source="train"`` the trainer recomputes behaviour log-probs itself. They must all be
taken from the weights the step started with -- before the first mini-batch's optimiser update -- or the
later mini-batches would see a ratio pinned at 1 and the clip / TIS bounds would never act. A tiny
fp32 model trains three mini-batches on CPU; what each mini-batch receives as its behaviour log-probs is
recorded and compared with log-probs computed up front from the starting weights.
"""

import random

import torch

from meshy_b200.backend.trainer import PPOTrainer
from meshy_b200.config import TrainerConfig, TrainerParamsConfig


def _batch(n=6, seed=3):
    rng = random.Random(seed)
    out = []
    for i in range(n):
        p, r = rng.randint(3, 9), rng.randint(5, 20)
        out.append({"tokens": torch.tensor([rng.randrange(2048) for _ in range(p + r)]),
                    "mask_assistant": torch.tensor([0] * p + [1] * r, dtype=torch.float32),
                    "logprobs": torch.tensor([0.0] * p + [-1.5] * r),
                    "advantage": torch.tensor([1.0 if i % 2 else -1.0]), "reward": torch.tensor([float(i % 2)]),
                    "weight_version": torch.tensor([0])})
    return out


def _trainer(source):
    tc = TrainerConfig(model_name="qwen3", model_flavor="debugmodel", seq_len=64, lr=3e-3, weight_decay=0.0,
                       max_norm=0.0, dtype="float32")
    tp = TrainerParamsConfig(mini_batch_size=2, batch_layout="packed", max_tokens_per_micro=64,
                             old_logprobs_source=source)
    return PPOTrainer(tc, tp, device="cpu", seed=1, timer_enabled=False)


def _record(trainer):
    seen = []
    inner = trainer._run_mini_batch

    def spy(samples, mini, timer, old_lps=None):
        seen.append(None if old_lps is None else [t.clone() for t in old_lps])
        return inner(samples, mini, timer, old_lps)

    trainer._run_mini_batch = spy
    return seen


def test_every_mini_batch_trains_against_the_starting_policy():
    t = _trainer("train")
    batch = _batch()
    full = t.plan_batch(batch, 1)
    local, plan = full.local_samples(batch, 0), full.per_rank[0]
    assert len(plan) == 3
    with torch.no_grad():
        start = [t.compute_old_logprobs(local, mini) for mini in plan]
    seen = _record(t)
    t.train_step(local, plan=plan)
    assert len(seen) == 3 and all(s is not None for s in seen)
    for want, got in zip(start, seen):
        for a, b in zip(want, got):
            assert torch.allclose(a, b, atol=1e-6)
    # the weights did move inside the step: the last mini-batch's log-probs under the final weights differ
    with torch.no_grad():
        after = t.compute_old_logprobs(local, plan[-1])
    assert max((a - b).abs().max().item() for a, b in zip(after, start[-1])) > 1e-4


def test_rollout_source_passes_no_recomputed_logprobs():
    t = _trainer("rollout")
    batch = _batch()
    seen = _record(t)
    t.train_step(batch)
    assert seen and all(s is None for s in seen)


def test_trainers_without_an_importance_ratio_skip_the_recompute():
    from meshy_b200.backend.opd import StudentTopKTrainer

    assert PPOTrainer.needs_behaviour_logprobs.fget(None) is True
    assert StudentTopKTrainer.needs_behaviour_logprobs.fget(None) is False
