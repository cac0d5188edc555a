"""Group-level advantage plug-ins (reference ``meshy/advantage.py`` and
``meshy/worker/rollout.py:88-97``)."""

from __future__ import annotations

import math
import os
from typing import Sequence

from .reward import response_length, soft_overlong_penalty


def grpo_advantage_values(rewards: Sequence[float]) -> list[float]:
    """``(r - mean) / max(std, 1e-8)`` over the group (unbiased std); a lone sample keeps its reward."""
    n = len(rewards)
    if n == 1:
        return [float(rewards[0])]
    mean = sum(rewards) / n
    var = sum((r - mean) ** 2 for r in rewards) / (n - 1)
    std = max(math.sqrt(var), 1e-8)
    return [(r - mean) / std for r in rewards]


def grpo_advantage(samples: list) -> None:
    """Write ``sample.advantage`` for a completed group (GRPO)."""
    for s, a in zip(samples, grpo_advantage_values([float(s.reward) for s in samples])):
        s.advantage = a


def is_zero_variance_group(samples: list, *, tolerance: float = 1e-8) -> bool:
    if not samples:
        return True
    r = [float(s.reward if getattr(s, "raw_reward", None) is None else s.raw_reward) for s in samples]
    return max(r) - min(r) <= tolerance


def _2_6_math_reshaped_advantage(samples: list, *, rollout_max_response_len: int = 126976,
                                 overlong_buffer_len: int | None = None, overlong_penalty_factor: float | None = None,
                                 length_reward_weight: float | None = None, length_reward_min_spread: int | None = None,
                                 length_reward_budget_floor: int | None = None) -> None:
    """DAPO soft-overlong shaping + optional length reward among correct samples, then group centering."""
    env = os.environ.get
    buf = int(env("OVERLONG_BUFFER_LEN", "25395")) if overlong_buffer_len is None else int(overlong_buffer_len)
    pf = float(env("OVERLONG_PENALTY_FACTOR", "1.0")) if overlong_penalty_factor is None else float(
        overlong_penalty_factor)
    lw = float(env("LENGTH_REWARD_WEIGHT", "0")) if length_reward_weight is None else float(length_reward_weight)
    spread_min = int(env("LENGTH_REWARD_MIN_SPREAD", "2000")) if length_reward_min_spread is None else int(
        length_reward_min_spread)
    floor = int(env("LENGTH_REWARD_BUDGET_FLOOR", "0")) if length_reward_budget_floor is None else int(
        length_reward_budget_floor)
    raw = [float(s.reward) for s in samples]
    lens = [response_length(s.masks) for s in samples]
    shaped = list(raw)
    if buf > 0:
        shaped = [soft_overlong_penalty(r, s, max_response_len=rollout_max_response_len, buffer_len=buf,
                                        penalty_factor=pf) for r, s in zip(shaped, samples)]
    if lw:
        correct = [i for i, r in enumerate(raw) if r > 0.5]
        if len(correct) >= 2:
            lo = min(lens[i] for i in correct)
            hi = max(lens[i] for i in correct)
            if hi - lo >= spread_min and hi >= floor:
                for i in correct:
                    shaped[i] += lw * (0.5 - (lens[i] - lo) / (hi - lo))
    mean = sum(shaped) / len(shaped)
    for s, r in zip(samples, shaped):
        s.advantage = r - mean


def assign_positive_lm_weights(group: list) -> None:
    """Group difficulty (1 - solve rate) as the positive-LM weight of correct binary-reward samples."""
    rewards = [float(s.reward if getattr(s, "raw_reward", None) is None else s.raw_reward) for s in group]
    binary = bool(rewards) and all(r in (0.0, 1.0) for r in rewards)
    difficulty = 1.0 - sum(rewards) / len(rewards) if binary else 0.0
    for s, r in zip(group, rewards):
        s.positive_lm_weight = difficulty if binary and r == 1.0 else 0.0


__all__ = ["_2_6_math_reshaped_advantage", "assign_positive_lm_weights", "grpo_advantage",
           "grpo_advantage_values", "is_zero_variance_group"]
