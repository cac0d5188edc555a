"""Group advantages and reward shaping (CPU): GRPO normalisation, the DAPO soft overlong penalty measured on the
first contiguous response span, group centering without std normalisation, the optional length reward among
correct samples, and the zero-variance group filter -- the same cases as the reference's rollout tests."""

from types import SimpleNamespace

import pytest

from meshy_b200.advantage import _2_6_math_reshaped_advantage, grpo_advantage, is_zero_variance_group
from meshy_b200.reward import response_length


def _samples(*rewards):
    return [SimpleNamespace(reward=r, advantage=None) for r in rewards]


def _masked(rewards, lengths, later_span=0):
    return [SimpleNamespace(reward=r, advantage=None, masks=[0, 0] + [1] * n + [0] + [1] * later_span)
            for r, n in zip(rewards, lengths)]


def test_grpo_default():
    s = _samples(1.0, 2.0, 3.0)
    grpo_advantage(s)
    assert [x.advantage for x in s] == pytest.approx([-1.0, 0.0, 1.0])


def test_response_length_first_span():
    assert response_length([0, 0, 1, 1, 1, 0, 1, 1]) == 3


def test_soft_overlong_penalty_and_centering():
    s = _masked([1.0, 0.0], [80, 100], later_span=50)
    _2_6_math_reshaped_advantage(s, rollout_max_response_len=100, overlong_buffer_len=20, overlong_penalty_factor=1.0,
                                 length_reward_weight=0.0)
    assert [x.advantage for x in s] == pytest.approx([1.0, -1.0])


def test_centering_without_std():
    s = _masked([1.0, 1.0, 0.0, 0.0], [10, 10, 10, 10])
    _2_6_math_reshaped_advantage(s, overlong_buffer_len=0, length_reward_weight=0.0)
    assert [x.advantage for x in s] == [0.5, 0.5, -0.5, -0.5]


def test_length_reward_among_correct():
    s = _masked([1.0, 1.0, 0.0], [10, 30, 20])
    _2_6_math_reshaped_advantage(s, overlong_buffer_len=0, length_reward_weight=0.2, length_reward_min_spread=1,
                                 length_reward_budget_floor=0)
    assert [x.advantage for x in s] == pytest.approx([1.1 - 2 / 3, 0.9 - 2 / 3, -2 / 3])


def test_zero_variance_filter():
    assert is_zero_variance_group(_samples(0.0, 0.0, 0.0))
    assert is_zero_variance_group(_samples(1.0, 1.0))
    assert not is_zero_variance_group(_samples(0.0, 1.0))
