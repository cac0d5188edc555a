"""Generalised advantage estimation (VAPO length-adaptive λ) and returns.

Definitions (reference ``meshy/backend/titan/critic/gae.py:70-312`` and
``trainer.py:603-699``), on the next-token grid, per ``[rows, S]`` block:

* ``cont_t = valid_t ∧ valid_{t+1} ∧ same_doc(t, t+1)`` links ``t → t+1``;
* ``δ_t = r_t + γ V_{t+1} cont_t − V_t`` on valid positions;
* ``A_t = δ_t + γ λ_doc cont_t A_{t+1}``;  ``G_t = r_t + γ cont_t G_{t+1}``;
* ``λ_doc = clamp(1 − 1/(α L_doc), 0, 1−1e-6)`` with ``L_doc`` the response
  length, or a constant ``gae_lambda``.

The recurrence is a segmented reverse *linear* recurrence.  On the GPU it is
one kernel (``gae_scan``): a block per row, a parallel scan over the affine
maps ``A ↦ x + d·A`` (associative), fp32 carries.  On the CPU it is the
sequential loop below in float64 vectorised over rows — the definition, and
the oracle for the kernel.
"""

from __future__ import annotations

import math

from typing import Any, Sequence

import numpy as np
import torch
import torch.distributed as dist

from ..ops.functional import native

ADVANTAGE_TOKENS = "advantage_tokens"


def lambda_per_doc(lengths: torch.Tensor, alpha: float, epsilon: float = 1e-6) -> torch.Tensor:
    L = lengths.clamp(min=1).float()
    return (1.0 - 1.0 / (alpha * L)).clamp(0.0, 1.0 - epsilon)


def continuation_mask(mask: torch.Tensor, doc_ids: torch.Tensor) -> torch.Tensor:
    valid = mask > 0
    cont = torch.zeros_like(valid)
    cont[:, :-1] = valid[:, :-1] & valid[:, 1:] & (doc_ids[:, 1:] == doc_ids[:, :-1])
    return cont.float()


def reverse_scan(x: torch.Tensor, decay: torch.Tensor, valid: torch.Tensor, cont: torch.Tensor) -> torch.Tensor:
    """``A_t = x_t + decay_t · cont_t · A_{t+1}`` (zero where not valid)."""
    if native(x):
        from ..ops._ext import ext

        out = torch.empty_like(x, dtype=torch.float32)
        ext().gae_scan(x.float().contiguous(), (decay * cont).float().contiguous(),
                       valid.float().contiguous(), out)
        return out
    xv = torch.where(valid, x, torch.zeros_like(x)).double().cpu().numpy()
    d = (decay * cont).double().cpu().numpy()
    rows, S = xv.shape
    out = np.zeros_like(xv)
    acc = np.zeros(rows)
    for t in range(S - 1, -1, -1):
        acc = xv[:, t] + d[:, t] * acc
        out[:, t] = acc
    res = torch.from_numpy(out).to(x.device, torch.float32)
    return torch.where(valid, res, torch.zeros_like(res))


def compute_returns(rewards, mask, doc_ids, *, gamma: float = 1.0) -> torch.Tensor:
    cont = continuation_mask(mask, doc_ids)
    return reverse_scan(rewards.float(), torch.full_like(rewards, float(gamma), dtype=torch.float32),
                        mask > 0, cont)


def compute_vapo_gae(rewards, values, mask, doc_ids, n_docs: int, *, lengths=None, gamma: float = 1.0,
                     alpha: float = 1.5, epsilon: float = 1e-6):
    rows, S = rewards.shape
    values = values.float()
    rewards = rewards.float()
    if lengths is None:
        cnt = torch.zeros(n_docs + 1, dtype=torch.float32, device=rewards.device).index_add_(
            0, doc_ids.reshape(-1), mask.reshape(-1).float())
        lengths = cnt[:n_docs]
    lam_doc = torch.cat([lambda_per_doc(lengths.to(rewards.device), alpha, epsilon), rewards.new_zeros(1)])
    lam = lam_doc[doc_ids]
    valid = mask > 0
    cont = continuation_mask(mask, doc_ids)
    next_v = torch.cat([values[:, 1:], values.new_zeros(rows, 1)], 1)
    delta = (rewards + gamma * next_v * cont - values) * valid.float()
    adv = reverse_scan(delta, gamma * lam, valid, cont)
    return adv, lam_doc[:n_docs]


def advantages_to_per_sequence(adv, mask, doc_ids, n_docs: int) -> torch.Tensor:
    flat = doc_ids.reshape(-1)
    s = adv.new_zeros(n_docs + 1).index_add_(0, flat, (adv * mask).reshape(-1))
    c = mask.new_zeros(n_docs + 1).index_add_(0, flat, mask.reshape(-1))
    return s[:n_docs] / c[:n_docs].clamp(min=1)


def attach_gae(samples: Sequence[Any], seq_len: int, *, gamma: float, alpha: float, lam: float | None,
               normalize: bool = False, group=None, device="cpu") -> dict[str, float]:
    """Per-token advantages from each row's ``values`` + ``reward`` columns."""
    if not samples:
        return {}
    rows = len(samples)
    widths = [min(int(len(td["tokens"])), seq_len) for td in samples]
    S = max(widths)
    mask = torch.zeros(rows, S)
    values = torch.zeros(rows, S)
    rewards = torch.zeros(rows, S)
    doc_ids = torch.arange(rows).unsqueeze(1).expand(rows, S).contiguous()
    for j, td in enumerate(samples):
        L = widths[j]
        m = torch.as_tensor(td["mask_assistant"][:L]).float()
        v = torch.as_tensor(td["values"][:L]).float()
        if v.shape[0] != L:
            raise ValueError(f"row {j}: {tuple(v.shape)} values for {L} tokens; critic and trainer disagree")
        mask[j, : L - 1] = m[1:L]
        values[j, :L] = v
        resp = (m > 0).nonzero()
        if resp.numel() == 0:
            continue
        last = int(resp[-1])
        if last == 0:
            continue
        rewards[j, last - 1] = float(torch.as_tensor(td["reward"]).reshape(-1)[0])
    if lam is None:
        a, lengths = alpha, None
    else:
        a, lengths = 1.0, torch.full((rows,), 1.0 / max(1e-9, 1.0 - lam))
    adv, lam_doc = compute_vapo_gae(rewards, values, mask, doc_ids, rows, gamma=gamma, alpha=a, lengths=lengths)
    if normalize:
        adv = whiten(adv, mask, group)
    for j, td in enumerate(samples):
        td[ADVANTAGE_TOKENS] = adv[j, : widths[j]].clone()
    n_tok = max(1.0, float(mask.sum()))
    per_seq = (adv * mask).sum(1) / mask.sum(1).clamp(min=1)
    return {
        "critic/value_mean": float((values * mask).sum() / n_tok),
        "critic/advantage_mean": float((adv * mask).sum() / n_tok),
        "critic/advantage_abs_mean": float((adv.abs() * mask).sum() / n_tok),
        "critic/advantage_seq_mean": float(per_seq.mean()),
        "critic/lambda_mean": float(lam_doc.mean()),
    }


def whiten(adv: torch.Tensor, mask: torch.Tensor, group=None, cp_degree: int = 1) -> torch.Tensor:
    """Whitening over the masked tokens of every rank of ``group``: ``(a - mean) / sqrt(var + 1e-8)`` with the
    unbiased variance (reference ``vapo.py:6-32``); unmasked tokens become 0. ``cp_degree``: ranks of the
    group that hold replicas of the same full sequences (CP ranks before sharding), counted once."""
    stats = torch.tensor([float((adv * mask).sum()), float((adv * adv * mask).sum()), float(mask.sum())],
                         dtype=torch.float64)
    if group is not None and dist.is_initialized() and dist.get_world_size(group) > 1:
        dev = torch.device("cuda") if dist.get_backend(group) == "nccl" else torch.device("cpu")
        st = stats.to(dev)
        dist.all_reduce(st, group=group)
        stats = st.cpu() / cp_degree
    s, s2, n = stats.tolist()
    count = max(n, 1.0)
    mean = s / count
    var = max(s2 / count - mean * mean, 0.0)
    if n >= 2:
        var *= n / (n - 1)
    return torch.where(mask > 0, (adv - mean) / math.sqrt(var + 1e-8), torch.zeros_like(adv))


__all__ = [
    "ADVANTAGE_TOKENS", "advantages_to_per_sequence", "attach_gae", "compute_returns", "compute_vapo_gae",
    "continuation_mask", "lambda_per_doc", "reverse_scan", "whiten",
]
