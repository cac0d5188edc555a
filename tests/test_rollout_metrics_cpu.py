"""Rollout metrics from the per-sample stamps, under the reference's tag names (CPU only).

Mirrors the reference's rollout-metrics check (``tests/test_rollout_metrics.py``): repetition, truncation
and mixed-version fractions come from the stamps the rollout worker ships; staleness is measured against the
trainer's current version; response lengths count assistant tokens only; rollout log-probs average over
sampled tokens only; without stamps the stamp tags are absent.
"""

import pytest
import torch

from meshy_b200.utils.metrics_adapter import rollout_metrics


def _sample(length=40, prompt=10, *, reward=1.0, version=3, truncated=False, repetition=False, mixed=False,
            seed=0):
    g = torch.Generator().manual_seed(seed)
    mask = torch.ones(length)
    mask[:prompt] = 0
    lp = -torch.rand(length, generator=g)
    lp[:prompt] = 0.0  # prompt placeholders
    return {"tokens": torch.randint(1, 1000, (length,), generator=g), "logprobs": lp, "mask_assistant": mask,
            "advantage": torch.tensor(0.5), "weight_version": torch.tensor(version), "reward": torch.tensor(reward),
            "truncated": torch.tensor(int(truncated)), "repetition": torch.tensor(int(repetition)),
            "mixed_version": torch.tensor(int(mixed))}


def test_rollout_metrics_use_stamps_and_rewards():
    samples = [
        _sample(reward=1.0, version=3, truncated=True, mixed=True, seed=1),
        _sample(reward=0.0, version=3, repetition=True, seed=2),
        _sample(reward=1.0, version=2, seed=3),
        _sample(reward=0.0, version=1, truncated=True, mixed=True, seed=4),
    ]
    m, hist = rollout_metrics(samples, seq_len=131072, current_version=4)
    assert m["rollout/truncated_ratio"] == pytest.approx(0.5)
    assert m["rollout/repetition_frac"] == pytest.approx(0.25)
    assert m["rollout/weight_version/mixed_version_ratio"] == pytest.approx(0.5)
    # two of the four samples are older than the newest version in the batch (3)
    assert m["rollout/weight_version/stale_ratio"] == pytest.approx(0.5)
    assert m["rollout/weight_version/max"] == 3 and m["rollout/weight_version/min"] == 1
    assert m["rollout/weight_version/num_versions"] == 3
    assert m["rollout/weight_version/mean"] == pytest.approx(9 / 4)
    assert m["rollout/weight_version/median"] == pytest.approx(2.5)
    assert m["rollout/weight_version/staleness_mean"] == pytest.approx((1 + 1 + 2 + 3) / 4)
    assert m["rollout/weight_version/staleness_max"] == 3
    assert m["rollout/raw_reward_mean"] == pytest.approx(0.5)
    assert m["rollout/rewards"] == pytest.approx(0.5)
    assert m["rollout/pass_rate"] == pytest.approx(0.5)
    assert m["rollout/response_len/mean"] == 30
    assert m["rollout/seq_len_truncated_ratio"] == 0.0
    assert m["rollout/log_probs"] < 0.0
    assert len(hist["rollout/log_probs"]) == 4 * 30


def test_rollout_metrics_without_stamps_omit_the_tags():
    plain = [{"tokens": torch.arange(20), "logprobs": -torch.ones(20), "mask_assistant": torch.ones(20),
              "advantage": torch.tensor(0.0), "weight_version": torch.tensor(0)}]
    m, _ = rollout_metrics(plain, seq_len=16)
    for tag in ("rollout/truncated_ratio", "rollout/repetition_frac", "rollout/weight_version/mixed_version_ratio",
                "rollout/raw_reward_mean"):
        assert tag not in m
    assert m["rollout/seq_len_truncated_ratio"] == 1.0
    assert m["rollout/log_probs"] == pytest.approx(-1.0)


def test_raw_reward_tags_read_the_unshaped_reward():
    """With shaping on, ``reward`` is shaped and ``raw_reward`` is not: the raw tags and the pass rate follow
    ``raw_reward``, ``rollout/rewards`` follows the shaped value."""
    samples = [_sample(reward=0.8, seed=5), _sample(reward=-0.3, seed=6)]
    samples[0]["raw_reward"] = torch.tensor(1.0)
    samples[1]["raw_reward"] = torch.tensor(0.0)
    m, _ = rollout_metrics(samples, current_version=3)
    assert m["rollout/raw_reward_mean"] == pytest.approx(0.5)
    assert m["rollout/raw_reward"] == pytest.approx(0.5)
    assert m["rollout/rewards"] == pytest.approx(0.25)
    assert m["rollout/pass_rate"] == pytest.approx(0.5)
    assert m["rollout/weight_version/stale_ratio"] == 0.0
