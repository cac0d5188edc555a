"""Micro-batch materialisation.

:func:`build_micro_batch` turns a :class:`~.plan.MicroPlan` plus the
rank-local samples into a :class:`Batch` on the device.  Same contract as the
reference (``meshy/backend/titan/batch.py:96-230``): next-token shift of labels,
mask and rollout log-probs inside each sample, a ``doc_ids`` companion (sample
index, ``n_docs`` for padding) for per-sequence reductions, and per-token or
per-sequence advantages.

Difference by design: both layouts are handed to the model as one packed
token stream with ``cu_seqlens``.  The padded layout ``[rows, S]`` becomes
``rows`` documents of length ``S`` (tail padding sits after the causal
frontier of every real token, so the result is identical), which lets one
varlen attention kernel serve both.  Per-document loss-token counts are
computed here on the host from the full sample, which removes the
context-parallel all-reduce of those counts.

Tensors are assembled in pinned host memory and copied with one
``non_blocking`` transfer each.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Sequence

import torch

from .plan import Layout, MicroPlan

ADVANTAGE_TOKENS = "advantage_tokens"


@dataclass
class Batch:
    input_ids: torch.Tensor          # [T] int64
    labels: torch.Tensor             # [T] int64 (shifted, pad 0)
    positions: torch.Tensor          # [T] int32
    mask: torch.Tensor               # [T] f32 (shifted assistant mask)
    doc_ids: torch.Tensor            # [T] int64 (n_docs = padding)
    advantages: torch.Tensor         # [n_docs] or [T] f32
    rollout_logprobs: torch.Tensor | None
    cu_seqlens: torch.Tensor         # [n_attn_docs + 1] int32
    max_seqlen: int
    n_docs: int
    seg_count: torch.Tensor          # [n_docs + 1] f32, global loss tokens per sample
    positive_lm_weights: torch.Tensor | None = None
    layout: Layout = "packed"
    rows: int = 1
    adv_per_token: bool = False
    h2d_bytes: int = 0
    extra: dict = field(default_factory=dict)

    @property
    def n_slots(self) -> int:
        return self.n_docs + 1

    @property
    def n_tokens(self) -> int:
        return int(self.input_ids.shape[0])


def _col(td: Any, name: str):
    v = td[name]
    return v if isinstance(v, torch.Tensor) else torch.as_tensor(v)


def _shift(x: torch.Tensor) -> torch.Tensor:
    return torch.cat([x[1:], x.new_zeros(1)])


def build_micro_batch(
    samples: Sequence[Any],
    micro: MicroPlan,
    *,
    layout: Layout,
    device: torch.device | str,
    need_rollout_lp: bool,
    sharder=None,
) -> Batch:
    n_docs = len(micro.sample_idx)
    per_token_adv = n_docs > 0 and ADVANTAGE_TOKENS in samples[micro.sample_idx[0]]
    pin = torch.device(device).type == "cuda"

    if layout == "padded":
        rows, S = micro.n_rows, micro.seq_len
        T = rows * S
        doc_starts = [j * S for j in range(rows)]
        cu = [j * S for j in range(rows + 1)]
        max_len = S
    else:
        T = micro.seq_len
        doc_starts = []
        off = 0
        for L in micro.doc_lens:
            doc_starts.append(off)
            off += L
        cu = doc_starts + [off]
        if T > off:
            cu.append(T)
        max_len = max(list(micro.doc_lens) + [T - off]) if T > 0 else 1
        rows = 1

    def buf(dtype, fill=0):
        t = torch.full((T,), fill, dtype=dtype)
        return t.pin_memory() if pin else t

    input_ids = buf(torch.long)
    labels = buf(torch.long)
    positions = buf(torch.int32)
    mask = buf(torch.float32)
    doc_ids = buf(torch.long, n_docs)
    rollout_lp = buf(torch.float32) if need_rollout_lp else None
    adv_tok = buf(torch.float32) if per_token_adv else None
    adv_seq = torch.zeros(n_docs, dtype=torch.float32)
    seg_count = torch.zeros(n_docs + 1, dtype=torch.float32)
    pos_w = torch.zeros(n_docs, dtype=torch.float32)

    for j, idx in enumerate(micro.sample_idx):
        td = samples[idx]
        L = micro.doc_lens[j]
        s = doc_starts[j]
        tok = _col(td, "tokens")[:L].long()
        m = _col(td, "mask_assistant")[:L].float()
        input_ids[s:s + L] = tok
        labels[s:s + L] = _shift(tok)
        sm = _shift(m)
        mask[s:s + L] = sm
        doc_ids[s:s + L] = j
        positions[s:s + L] = torch.arange(L, dtype=torch.int32)
        seg_count[j] = float((sm > 0).sum())
        if rollout_lp is not None:
            rollout_lp[s:s + L] = _shift(_col(td, "logprobs")[:L].float())
        if adv_tok is not None:
            adv_tok[s:s + L] = _col(td, ADVANTAGE_TOKENS)[:L].float()
        else:
            adv_seq[j] = float(_col(td, "advantage").reshape(-1)[0]) if "advantage" in td else 0.0
        reward = float(_col(td, "reward").reshape(-1)[0]) if "reward" in td else 0.0
        if reward > 0.5 and "positive_lm_weight" in td:
            pos_w[j] = float(_col(td, "positive_lm_weight").reshape(-1)[0])

    if layout == "padded":
        # positions restart per row; tail padding keeps counting (never attended by real tokens)
        positions.copy_(torch.arange(S, dtype=torch.int32).repeat(rows))
        if n_docs == 0:
            doc_ids.fill_(0)
    elif T > (cu[len(micro.doc_lens)] if micro.doc_lens else 0):
        off = cu[len(micro.doc_lens)]
        positions[off:] = torch.arange(T - off, dtype=torch.int32)

    dev = torch.device(device)
    nb = dev.type == "cuda"
    h2d = 0

    def to(t):
        nonlocal h2d
        if t is None:
            return None
        h2d += t.numel() * t.element_size()
        return t.to(dev, non_blocking=nb)

    batch = Batch(
        input_ids=to(input_ids),
        labels=to(labels),
        positions=to(positions),
        mask=to(mask),
        doc_ids=to(doc_ids),
        advantages=to(adv_tok) if adv_tok is not None else to(adv_seq),
        rollout_logprobs=to(rollout_lp),
        cu_seqlens=to(torch.tensor(cu, dtype=torch.int32)),
        max_seqlen=int(max_len),
        n_docs=n_docs,
        seg_count=to(seg_count),
        positive_lm_weights=to(pos_w),
        layout=layout,
        rows=rows,
        adv_per_token=adv_tok is not None,
    )
    batch.h2d_bytes = h2d
    if sharder is not None:
        batch = sharder.shard_batch(batch)
    return batch


__all__ = ["ADVANTAGE_TOKENS", "Batch", "build_micro_batch"]
