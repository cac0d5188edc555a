"""Per-sample reward shaping (reference ``meshy/reward.py:33-92``).

Signature of every shaping rule: ``fn(reward, sample, **kwargs) -> float``.
Shaping belongs to the reward, not the advantage estimator, so it applies the
same way under a group baseline and under an external critic.
"""

from __future__ import annotations

import os
from typing import Any, Iterable


def response_length(mask: Iterable[float]) -> int:
    """Length of the first contiguous run of response tokens in ``mask``."""
    n, started = 0, False
    for v in mask:
        if v:
            started = True
            n += 1
        elif started:
            break
    return n


def soft_overlong_penalty(reward: float, sample: Any, *, max_response_len: int = 126976,
                          buffer_len: int | None = None, penalty_factor: float | None = None) -> float:
    """DAPO soft length penalty: linear ramp to ``-penalty_factor`` over the last ``buffer_len`` tokens."""
    buffer_len = int(os.environ.get("OVERLONG_BUFFER_LEN", "25395")) if buffer_len is None else int(buffer_len)
    penalty_factor = (float(os.environ.get("OVERLONG_PENALTY_FACTOR", "1.0")) if penalty_factor is None
                      else float(penalty_factor))
    if buffer_len <= 0:
        return float(reward)
    length = response_length(getattr(sample, "masks", None) or sample["mask_assistant"])
    expected = int(max_response_len) - buffer_len
    if length <= expected:
        return float(reward)
    return float(reward) + max((expected - length) / buffer_len * penalty_factor, -penalty_factor)


__all__ = ["response_length", "soft_overlong_penalty"]
