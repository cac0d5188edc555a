"""CPU tests of the training semantics (BASELINE config 1 building blocks)."""

import math
import random

import pytest
import torch

from meshy_b200.advantage import grpo_advantage_values
from meshy_b200.backend import gae
from meshy_b200.backend.batch import build_micro_batch
from meshy_b200.backend.loss import LossConfig, ppo_clip_loss
from meshy_b200.backend.plan import PlannerConfig, build_plan, plan_stats, resolve_align, snake_deal


def test_snake_deal():
    assert snake_deal(list(range(7)), 3) == [[0, 5, 6], [1, 4], [2, 3]]


@pytest.mark.parametrize("layout", ["padded", "packed"])
def test_plan_invariants(layout):
    rng = random.Random(0)
    lengths = [rng.randint(5, 300) for _ in range(24)]
    loss_tok = [max(0, L - 3) for L in lengths]
    cfg = PlannerConfig(layout=layout, mini_batch_size=3, seq_len=256, align=16, max_tokens_per_micro=512)
    plan = build_plan(lengths, loss_tok, 4, cfg)
    assert plan.dp_size == 4
    seen = sorted(i for r in plan.local_indices for i in r)
    assert seen == list(range(24))
    for i in range(len(plan.per_rank[0])):
        counts = {len(plan.per_rank[r][i].micros) for r in range(4)}
        assert len(counts) == 1
        assert len({plan.per_rank[r][i].n_docs_global for r in range(4)}) == 1
    for r in range(4):
        for mini in plan.per_rank[r]:
            for m in mini.micros:
                if m.is_filler:
                    continue
                cost = m.n_rows * m.seq_len if layout == "padded" else m.seq_len
                assert cost <= 512 or len(m.sample_idx) == 1
    st = plan_stats(plan.per_rank[0], layout)
    assert 0 <= st["padding_ratio"] < 1
    assert resolve_align(2048, 8, 16384) == 2048


def test_grpo_advantage():
    a = grpo_advantage_values([1.0, 0.0, 1.0, 0.0])
    assert abs(sum(a)) < 1e-6 and abs(a[0] - 0.8660254) < 1e-5
    assert grpo_advantage_values([3.0]) == [3.0]


def _batch(samples, layout="packed"):
    from meshy_b200.backend.plan import MicroPlan

    lens = tuple(len(s["tokens"]) for s in samples)
    seq = sum(lens) if layout == "packed" else max(lens)
    micro = MicroPlan(tuple(range(len(samples))), seq, lens)
    return build_micro_batch(samples, micro, layout=layout, device="cpu", need_rollout_lp=True)


def _samples(n=3):
    out = []
    for i in range(n):
        L = 10 + 3 * i
        m = torch.zeros(L)
        m[4:] = 1
        out.append({"tokens": torch.arange(L) + i, "mask_assistant": m, "logprobs": -torch.rand(L),
                    "advantage": torch.tensor(float(i) - 1), "reward": torch.tensor(1.0)})
    return out


def test_micro_batch_shift_and_layouts():
    s = _samples()
    for layout in ("packed", "padded"):
        b = _batch(s, layout)
        assert b.n_docs == 3
        if layout == "packed":
            assert b.cu_seqlens.tolist() == [0, 10, 23, 39]
            assert torch.equal(b.labels[:9], s[0]["tokens"][1:10])
            assert b.labels[9] == 0 and b.mask[9] == 0
            assert b.mask[:10].sum() == 6
        assert b.seg_count[:3].tolist() == [6.0, 9.0, 12.0]


def test_ppo_loss_sequence_mean_and_grad():
    s = _samples()
    b = _batch(s)
    old = b.rollout_logprobs.clone()
    new = (old + 0.1 * torch.randn_like(old)).requires_grad_(True)
    loss, sums = ppo_clip_loss(new, old, b, 3, 27, LossConfig(0.2, 0.28))
    # reference formula written out per document
    r = torch.exp(new.detach() - old)
    adv = torch.cat([b.advantages, torch.zeros(1)])[b.doc_ids]
    pg = -torch.minimum(r * adv, r.clamp(0.8, 1.28) * adv) * b.mask
    expect = sum((pg[b.doc_ids == d].sum() / b.mask[b.doc_ids == d].sum()) for d in range(3)) / 3
    assert abs(loss.item() - expect.item()) < 1e-6
    loss.backward()
    assert torch.isfinite(new.grad).all()
    assert sums["token_count"].item() == 27


def test_gae_constant_lambda_matches_definition():
    torch.manual_seed(0)
    rows, S = 2, 50
    mask = torch.zeros(rows, S)
    mask[0, 5:40] = 1
    mask[1, 0:50] = 1
    doc = torch.arange(rows).unsqueeze(1).expand(rows, S).contiguous()
    r = torch.zeros(rows, S)
    r[0, 39] = 1.0
    r[1, 49] = -1.0
    v = torch.randn(rows, S) * 0.1
    adv, lam = gae.compute_vapo_gae(r, v, mask, doc, rows, gamma=1.0, alpha=1.0,
                                    lengths=torch.full((rows,), 1 / (1 - 0.95)))
    assert torch.allclose(lam, torch.full((rows,), 0.95), atol=1e-5)
    # direct recursion
    for row in range(rows):
        A = 0.0
        for t in range(S - 1, -1, -1):
            if mask[row, t] == 0:
                A = 0.0
                continue
            cont = 1.0 if (t + 1 < S and mask[row, t + 1] > 0) else 0.0
            delta = r[row, t] + cont * v[row, t + 1 if t + 1 < S else t] - v[row, t]
            A = delta + 0.95 * cont * A
            assert abs(adv[row, t].item() - A) < 1e-4
    ret = gae.compute_returns(r, mask, doc)
    assert ret[0, 5].item() == pytest.approx(1.0) and ret[1, 0].item() == pytest.approx(-1.0)
