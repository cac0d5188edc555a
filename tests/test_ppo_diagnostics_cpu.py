"""PPO loss diagnostics on the CPU path: ``ppo_kl``, ``train_rollout_kl``, ``ess_ratio``, entropy.

Mirrors the reference's diagnostics check (``tests/test_ppo_diagnostics.py``): a constant log-ratio gives a
k1 KL of ``-delta``, a ratio of ``exp(delta)``, a full effective sample size and a k3 KL between the rollout
and the trainer of ``exp(-delta) + delta - 1``; one heavy token per sequence lowers the ESS below 1; without
rollout log-probs the train/rollout KL is not reported; the diagnostics leave autograd intact.
"""

import math

import pytest
import torch

from meshy_b200.backend.batch import Batch
from meshy_b200.backend.loss import LossConfig, ppo_clip_loss, reduce_sums


def _batch(rows=2, S=8, rollout=None):
    """``rows`` packed documents of ``S`` tokens each; the last token of every document carries no loss."""
    T = rows * S
    mask = torch.ones(rows, S)
    mask[:, -1] = 0
    doc_ids = torch.arange(rows).repeat_interleave(S)
    return Batch(
        input_ids=torch.zeros(T, dtype=torch.long), labels=torch.zeros(T, dtype=torch.long),
        positions=torch.arange(S, dtype=torch.int32).repeat(rows), mask=mask.reshape(T), doc_ids=doc_ids,
        advantages=torch.tensor([1.0, -1.0])[:rows], rollout_logprobs=rollout,
        cu_seqlens=torch.arange(rows + 1, dtype=torch.int32) * S, max_seqlen=S, n_docs=rows,
        seg_count=torch.cat([mask.sum(1), torch.zeros(1)]),
    )


def test_constant_log_ratio_reports_kl_ratio_and_full_ess():
    old = -torch.ones(16)
    delta = 0.1
    new = (old + delta).requires_grad_()
    b = _batch(rollout=old.clone())
    loss, sums = ppo_clip_loss(new, old, b, 2, int(b.mask.sum()),
                               LossConfig(0.2, 0.28, use_tis=True), entropy=torch.full((16,), 2.0))
    red = reduce_sums(sums)
    assert red["ppo_kl"] == pytest.approx(-delta)
    assert red["log_ratio_abs_mean"] == pytest.approx(delta)
    assert red["ratio_mean"] == pytest.approx(math.exp(delta))
    assert red["ess_ratio"] == pytest.approx(1.0)
    assert red["entropy"] == pytest.approx(2.0)
    assert red["train_rollout_kl"] == pytest.approx(math.exp(-delta) + delta - 1, rel=1e-4)
    assert red["train_rollout_logdiff_abs"] == pytest.approx(delta)
    assert sums["token_count"].item() == float(b.mask.sum())
    loss.backward()
    assert new.grad is not None and torch.isfinite(new.grad).all()


def test_uneven_weights_lower_ess_and_no_rollout_kl_without_rollout_logprobs():
    old = torch.zeros(16)
    new = torch.zeros(16)
    new[0] = new[8] = 1.5  # one heavy token per sequence
    b = _batch()
    _, sums = ppo_clip_loss(new, old, b, 2, int(b.mask.sum()), LossConfig(0.2, 0.28, use_tis=True))
    red = reduce_sums(sums)
    assert 0.0 < red["ess_ratio"] < 1.0
    # ESS of one sequence written out: (sum w)^2 / (n sum w^2) over its 7 loss tokens
    w = torch.ones(7)
    w[0] = math.exp(1.5)
    assert red["ess_ratio"] == pytest.approx((w.sum() ** 2 / (7 * (w * w).sum())).item(), rel=1e-5)
    assert "train_rollout_kl" not in red and "entropy" not in red


def test_tis_drops_tokens_outside_the_band():
    old = torch.zeros(16)
    new = torch.zeros(16)
    new[1] = 2.0  # ratio e^2 > 5: dropped
    new[2] = -1.0  # ratio e^-1 < 0.5: dropped
    b = _batch()
    _, sums = ppo_clip_loss(new, old, b, 2, int(b.mask.sum()), LossConfig(0.2, 0.28, use_tis=True))
    red = reduce_sums(sums)
    assert red["tis_masked_frac"] == pytest.approx(2 / 14)
    assert red["clip_frac"] == pytest.approx(2 / 14)
