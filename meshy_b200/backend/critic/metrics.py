"""Critic health gauges (reference ``meshy/backend/titan/critic/metrics.py:58-322``).

All gauges use ``V0``, the predicted value of the state right before the
first response token (the critic's estimate of the prompt's solve rate), and
the sample's reward ``R``:

* ``prompt_pearson`` — Pearson correlation over prompts of mean ``V0`` vs mean
  ``R`` (does the critic rank prompts by difficulty?);
* ``within_prompt_auc`` — over pairs of samples of one prompt with different
  rewards, the fraction the critic orders correctly by their ``V0`` after the
  first response token (ties count half);
* ``variance_reduction`` — ``1 - Var(R - V0) / Var(R)``, the share of reward
  variance the baseline explains;
* ``calibration_gap`` — ``|mean V0 - mean R|``.

:class:`StreamingGauges` accumulates the sums across windows so the gauges
cover more than one window's rows.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Sequence


def _mean(x: Sequence[float]) -> float:
    return sum(x) / len(x) if x else float("nan")


def prompt_pearson(v0: Sequence[float], rewards: Sequence[float], groups: Sequence[Sequence[int]]) -> float:
    mv = [_mean([v0[i] for i in g]) for g in groups]
    mr = [_mean([rewards[i] for i in g]) for g in groups]
    if len(mv) < 2:
        return float("nan")
    a, b = _mean(mv), _mean(mr)
    cov = sum((x - a) * (y - b) for x, y in zip(mv, mr))
    va = sum((x - a) ** 2 for x in mv)
    vb = sum((y - b) ** 2 for y in mr)
    if va <= 0 or vb <= 0:
        return float("nan")
    return cov / math.sqrt(va * vb)


def within_prompt_auc(v_first: Sequence[float], rewards: Sequence[float], groups: Sequence[Sequence[int]]) -> float:
    good = total = 0.0
    for g in groups:
        for x in range(len(g)):
            for y in range(x + 1, len(g)):
                i, j = g[x], g[y]
                if rewards[i] == rewards[j]:
                    continue
                hi, lo = (i, j) if rewards[i] > rewards[j] else (j, i)
                total += 1
                if v_first[hi] > v_first[lo]:
                    good += 1
                elif v_first[hi] == v_first[lo]:
                    good += 0.5
    return good / total if total else float("nan")


def variance_reduction(v0: Sequence[float], rewards: Sequence[float]) -> float:
    if len(rewards) < 2:
        return float("nan")
    mr = _mean(rewards)
    var_r = _mean([(r - mr) ** 2 for r in rewards])
    res = [r - v for r, v in zip(rewards, v0)]
    m = _mean(res)
    var_res = _mean([(x - m) ** 2 for x in res])
    return 1.0 - var_res / var_r if var_r > 0 else float("nan")


def calibration_gap(v0: Sequence[float], rewards: Sequence[float]) -> float:
    return abs(_mean(v0) - _mean(rewards))


@dataclass
class CriticDiagnostics:
    prompt_pearson: float
    within_prompt_auc: float
    variance_reduction: float
    calibration_gap: float
    n: int

    def as_dict(self) -> dict[str, float]:
        return {f"critic/{k}": float(v) for k, v in self.__dict__.items()}

    def __str__(self) -> str:
        return (f"pearson={self.prompt_pearson:.3f} auc={self.within_prompt_auc:.3f} "
                f"var_red={self.variance_reduction:.3f} calib={self.calibration_gap:.3f} n={self.n}")


def critic_diagnostics(v0, v_first, rewards, groups) -> CriticDiagnostics:
    return CriticDiagnostics(prompt_pearson(v0, rewards, groups), within_prompt_auc(v_first, rewards, groups),
                             variance_reduction(v0, rewards), calibration_gap(v0, rewards), len(rewards))


class StreamingGauges:
    """Running sums for the variance-reduction and calibration gauges across windows."""

    def __init__(self):
        self.n = 0
        self.sr = self.sr2 = self.sv = self.sres = self.sres2 = 0.0

    def update(self, v0: Sequence[float], rewards: Sequence[float]) -> None:
        for v, r in zip(v0, rewards):
            self.n += 1
            self.sr += r
            self.sr2 += r * r
            self.sv += v
            self.sres += r - v
            self.sres2 += (r - v) ** 2

    def as_dict(self) -> dict[str, float]:
        if self.n < 2:
            return {}
        var_r = self.sr2 / self.n - (self.sr / self.n) ** 2
        var_res = self.sres2 / self.n - (self.sres / self.n) ** 2
        return {"critic/stream_variance_reduction": 1 - var_res / var_r if var_r > 0 else float("nan"),
                "critic/stream_calibration_gap": abs(self.sv / self.n - self.sr / self.n), "critic/stream_n": self.n}


__all__ = ["CriticDiagnostics", "StreamingGauges", "calibration_gap", "critic_diagnostics", "prompt_pearson",
           "variance_reduction", "within_prompt_auc"]
