"""CPU numerics of the distillation loss and the critic pieces against direct definitions."""

import math
import random

import torch

from meshy_b200.backend.critic.data import TrajectorySample, pack_micros, row_targets, split_by_prompt
from meshy_b200.backend.critic.metrics import (calibration_gap, prompt_pearson, variance_reduction,
                                               within_prompt_auc)
from meshy_b200.backend.topk_loss import forward_kl_topk, gather_logprobs, teacher_topk
from meshy_b200.backend.vapo import clipped_value_error
from meshy_b200.utils.metrics_adapter import MetricsWriter, crc32c, read_events, rollout_metrics


def test_topk_pipeline_matches_dense_definition():
    torch.manual_seed(0)
    T, D, V, K = 37, 16, 50, 5
    h, w = torch.randn(T, D), torch.randn(V, D)
    ids, lps = teacher_topk(h, w, K, chunk=8)
    z = h @ w.t()
    ref_lp = torch.log_softmax(z, -1)
    top = ref_lp.topk(K, -1)
    assert torch.equal(ids, top.indices) and torch.allclose(lps, top.values, atol=1e-5)
    h2 = h.clone().requires_grad_(True)
    s = gather_logprobs(h2, w, ids, chunk=8)
    assert torch.allclose(s, ref_lp.gather(-1, ids), atol=1e-5)
    kl = forward_kl_topk(s, lps * 0.5, log_prob_min_clamp=-10.0, loss_max_clamp=10.0)
    t = (lps * 0.5).clamp_min(-10)
    want = (t.exp() * (t - s.clamp_min(-10))).sum(-1).clamp(-10, 10)
    assert torch.allclose(kl, want, atol=1e-6)
    kl.sum().backward()
    assert h2.grad is not None and torch.isfinite(h2.grad).all()


def test_clipped_value_error():
    v, r, old = torch.tensor([1.0, 0.0]), torch.tensor([0.0, 1.0]), torch.tensor([0.5, 0.5])
    got = clipped_value_error(v, r, old, 0.2)
    # clipped values 0.7 / 0.3 → errors max(1, 0.49) = 1, max(1, 0.49) = 1
    assert torch.allclose(got, torch.tensor([1.0, 1.0]))
    assert torch.allclose(clipped_value_error(v, r, None, None), torch.tensor([1.0, 1.0]))


def test_critic_targets_and_packing():
    s = TrajectorySample([5, 6, 7, 8, 9], [0, 0, 1, 1, 1], 1.0)
    mask, ret = row_targets(s, 16, gamma=0.5)
    assert mask.tolist() == [0, 1, 1, 1, 0]
    assert ret.tolist() == [0, 0.25, 0.5, 1.0, 0]
    samples = [TrajectorySample([1] * n, [0] * 2 + [1] * (n - 2), 0.0) for n in (10, 7, 12, 3, 9)]
    micros = pack_micros(samples, range(5), 64, 20)
    assert sorted(r for m in micros for r in m.rows) == list(range(5))
    assert all(int(m.cu_seqlens[-1]) <= 20 for m in micros)


def test_critic_gauges():
    groups = split_by_prompt([TrajectorySample([1, 2, 9], [0, 0, 1], 1.0), TrajectorySample([1, 2, 8], [0, 0, 1], 0.0),
                              TrajectorySample([3, 9], [0, 1], 1.0)])
    assert groups == [[0, 1], [2]]
    v, r = [0.9, 0.1, 0.8], [1.0, 0.0, 1.0]
    assert within_prompt_auc(v, r, groups) == 1.0
    assert math.isclose(calibration_gap(v, r), abs(sum(v) / 3 - 2 / 3))
    assert variance_reduction(r, r) == 1.0
    assert not math.isnan(prompt_pearson([0.1, 0.2, 0.9], [0.0, 0.0, 1.0], [[0], [1], [2]]))


def test_event_writer_roundtrip(tmp_path):
    assert crc32c(b"123456789") == 0xE3069283  # the CRC-32C check value
    w = MetricsWriter(str(tmp_path), use_tensorboard=False)
    w.write({"a": 1.5, "b": 2}, 7, {"x": [1.0, 2.0, 3.0]})
    w.close()
    ev = [f for f in tmp_path.iterdir() if f.name.startswith("events.out")][0]
    recs = read_events(str(ev))
    assert recs[-1] == (7, {"a": 1.5, "b": 2.0})


def test_rollout_metrics():
    rng = random.Random(0)
    rows = [{"tokens": list(range(10 + i)), "mask_assistant": [0] * 5 + [1] * (5 + i), "reward": float(i % 2),
             "advantage": [0.5 - (i % 2)], "weight_version": 3, "truncated": i == 0, "repetition": False,
             "mixed_version": False} for i in range(6)]
    m, h = rollout_metrics(rows, seq_len=12, current_version=4)
    assert m["rollout/pass_rate"] == 0.5
    assert m["rollout/truncated_ratio"] == 1 / 6
    assert m["rollout/staleness/mean"] == 1.0
    assert m["rollout/response_len/max"] == 10
    assert len(h["response_length"]) == 6
    del rng
