"""Advantage estimators and reward shaping, checked against the formulas they implement (CPU).

* GRPO: ``(r - mean) / std`` with the unbiased std over the group; invariant to shifting the rewards,
  zero-mean, unit sample variance; a constant group gets all-zero advantages; a lone sample keeps its reward.
* DAPO soft overlong penalty: no change up to ``max_len - buffer``, then a linear ramp to ``-factor`` at
  ``max_len`` and flat beyond; the length is that of the *first* response span of the mask.
* ``_2_6_math`` shaping: shaped rewards are centred (no std), the optional length bonus ranks only correct
  samples, and needs a minimum length spread.
"""

import math
import random
from types import SimpleNamespace

import pytest

from meshy_b200.advantage import (_2_6_math_reshaped_advantage, grpo_advantage, grpo_advantage_values,
                                  is_zero_variance_group)
from meshy_b200.reward import response_length, soft_overlong_penalty


def _resp(reward, n_resp, prompt=5, tail=0):
    """A sample whose mask has a ``prompt`` prefix, ``n_resp`` response tokens, a gap, and ``tail`` more."""
    return SimpleNamespace(reward=reward, advantage=None, masks=[0] * prompt + [1] * n_resp + [0, 0] + [1] * tail)


@pytest.mark.parametrize("seed", range(5))
def test_grpo_is_a_standardisation(seed):
    rng = random.Random(seed)
    r = [rng.uniform(-3, 3) for _ in range(rng.randint(2, 12))]
    a = grpo_advantage_values(r)
    n = len(a)
    assert sum(a) == pytest.approx(0.0, abs=1e-9)
    assert sum(x * x for x in a) / (n - 1) == pytest.approx(1.0, rel=1e-9)
    assert grpo_advantage_values([x + 10.0 for x in r]) == pytest.approx(a)
    # order preserving
    assert sorted(range(n), key=lambda i: r[i]) == sorted(range(n), key=lambda i: a[i])


def test_grpo_degenerate_groups():
    assert grpo_advantage_values([0.7, 0.7, 0.7]) == pytest.approx([0.0, 0.0, 0.0], abs=1e-6)
    assert grpo_advantage_values([0.3]) == [0.3]
    group = [SimpleNamespace(reward=v, advantage=None) for v in (0.0, 1.0, 1.0, 0.0)]
    grpo_advantage(group)
    expected = 0.5 / math.sqrt(1.0 / 3.0)
    assert [g.advantage for g in group] == pytest.approx([-expected, expected, expected, -expected])


def test_response_length_counts_only_the_first_span():
    assert response_length([0, 1, 1, 0, 1]) == 2
    assert response_length([1, 1, 1]) == 3
    assert response_length([0, 0]) == 0


@pytest.mark.parametrize("length,want", [(60, 1.0), (70, 1.0), (75, 0.75), (90, 0.0), (200, 0.0)])
def test_soft_overlong_penalty_ramp(length, want):
    # max 90, buffer 20: free up to 70, then -1/20 per token, floor at -1 (reward 1 -> 0)
    s = _resp(1.0, length, tail=40)  # the tail span after the gap must not count
    assert soft_overlong_penalty(1.0, s, max_response_len=90, buffer_len=20, penalty_factor=1.0) == pytest.approx(want)


def test_reshaped_advantage_is_centred_not_scaled():
    group = [_resp(1.0, 10), _resp(1.0, 12), _resp(0.0, 9), _resp(0.0, 30), _resp(0.0, 7)]
    _2_6_math_reshaped_advantage(group, overlong_buffer_len=0, length_reward_weight=0.0)
    assert [g.advantage for g in group] == pytest.approx([0.6, 0.6, -0.4, -0.4, -0.4])


def test_reshaped_advantage_applies_the_overlong_penalty_first():
    # max 100, buffer 40: free up to 60 tokens; 90 tokens -> (60 - 90) / 40 = -0.75; shaped 0.25 and 1.0
    group = [_resp(1.0, 90), _resp(1.0, 20)]
    _2_6_math_reshaped_advantage(group, rollout_max_response_len=100, overlong_buffer_len=40,
                                 overlong_penalty_factor=1.0, length_reward_weight=0.0)
    assert [g.advantage for g in group] == pytest.approx([-0.375, 0.375])


def test_length_bonus_ranks_correct_samples_only():
    # correct lengths 40 and 100: bonus w * (0.5 - (L - 40) / 60) = +0.15 / -0.15 with w = 0.3
    group = [_resp(1.0, 40), _resp(1.0, 100), _resp(0.0, 10)]
    _2_6_math_reshaped_advantage(group, overlong_buffer_len=0, length_reward_weight=0.3,
                                 length_reward_min_spread=10, length_reward_budget_floor=0)
    shaped = [1.15, 0.85, 0.0]
    mean = sum(shaped) / 3
    assert [g.advantage for g in group] == pytest.approx([v - mean for v in shaped])
    # below the minimum spread the bonus is off
    group = [_resp(1.0, 40), _resp(1.0, 45), _resp(0.0, 10)]
    _2_6_math_reshaped_advantage(group, overlong_buffer_len=0, length_reward_weight=0.3,
                                 length_reward_min_spread=10, length_reward_budget_floor=0)
    assert [g.advantage for g in group] == pytest.approx([1 / 3, 1 / 3, -2 / 3])


def test_zero_variance_groups_are_detected_on_raw_rewards():
    same = [SimpleNamespace(reward=0.2, raw_reward=1.0), SimpleNamespace(reward=0.9, raw_reward=1.0)]
    assert is_zero_variance_group(same)  # shaping differences do not count
    mixed = [SimpleNamespace(reward=1.0, raw_reward=None), SimpleNamespace(reward=0.0, raw_reward=None)]
    assert not is_zero_variance_group(mixed)
    assert is_zero_variance_group([])
