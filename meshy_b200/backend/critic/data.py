"""Critic window data: rows → per-token tensors, prompt groups and packed micro-batches.

Semantics of the reference's critic data helpers
(``meshy/backend/titan/critic/data.py:69-351``): each row's ``mask_assistant``
marks response tokens; on the next-token grid the state at position ``t`` is
the prefix ``tokens[:t+1]`` and the action is ``tokens[t+1]``, so the shifted
mask is ``m[1:]``, the terminal reward sits on the last shifted response
position, and the value target at ``t`` is the return ``G_t``
(``compute_returns``).  Rows of one prompt share the prompt prefix, which
:func:`split_by_prompt` uses to group them.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Sequence

import torch


@dataclass
class TrajectorySample:
    tokens: list[int]
    mask: list[float]
    reward: float
    weight_version: int = 0

    @property
    def n_response(self) -> int:
        return int(sum(1 for m in self.mask if m))

    @property
    def prompt_key(self) -> tuple[int, ...]:
        out = []
        for t, m in zip(self.tokens, self.mask):
            if m:
                break
            out.append(int(t))
        return tuple(out)


def _list(x) -> list:
    return torch.as_tensor(x).reshape(-1).tolist()


def sample_from_row(row: Any) -> TrajectorySample:
    get = row.get if isinstance(row, dict) else (lambda k, d=None: getattr(row, k, d))
    reward = float(_list(get("reward"))[0])
    wv = get("weight_version", 0)
    wv = int(_list(wv)[0]) if wv is not None else 0
    return TrajectorySample([int(t) for t in _list(get("tokens"))], [float(m) for m in _list(get("mask_assistant"))],
                            reward, wv)


def samples_from_rows(rows: Sequence[Any]) -> list[TrajectorySample]:
    return [sample_from_row(r) for r in rows]


def split_by_prompt(samples: Sequence[TrajectorySample]) -> list[list[int]]:
    """Indices grouped by shared prompt prefix, in first-appearance order."""
    groups: dict[tuple[int, ...], list[int]] = {}
    for i, s in enumerate(samples):
        groups.setdefault(s.prompt_key, []).append(i)
    return list(groups.values())


def row_targets(s: TrajectorySample, seq_len: int, gamma: float = 1.0) -> tuple[torch.Tensor, torch.Tensor]:
    """Shifted response mask and return targets ``[L]`` of one row (``L = min(len, seq_len)``)."""
    L = min(len(s.tokens), seq_len)
    m = torch.tensor(s.mask[:L], dtype=torch.float32)
    mask = torch.zeros(L)
    if L > 1:
        mask[: L - 1] = m[1:L]
    ret = torch.zeros(L)
    resp = (mask > 0).nonzero().flatten()
    if resp.numel():
        last = int(resp[-1])
        # G_t = r_T gamma^(T - t) on the contiguous response span
        g = s.reward
        for t in range(last, -1, -1):
            if mask[t] <= 0:
                break
            ret[t] = g
            g *= gamma
    return mask, ret


@dataclass
class CriticMicro:
    rows: list[int]
    input_ids: torch.Tensor   # [T]
    positions: torch.Tensor   # [T] int32
    cu_seqlens: torch.Tensor  # [n + 1] int32
    max_seqlen: int
    mask: torch.Tensor        # [T]
    returns: torch.Tensor     # [T]
    lengths: list[int]


def pack_micros(samples: Sequence[TrajectorySample], rows: Sequence[int], seq_len: int, max_tokens: int | None,
                gamma: float = 1.0) -> list[CriticMicro]:
    """First-fit-decreasing packing of ``rows`` into micro-batches of at most ``max_tokens`` tokens."""
    lens = {i: min(len(samples[i].tokens), seq_len) for i in rows}
    order = sorted(rows, key=lambda i: (-lens[i], i))
    budget = max_tokens or sum(lens.values())
    bins: list[list[int]] = []
    loads: list[int] = []
    for i in order:
        for b, load in enumerate(loads):
            if load + lens[i] <= budget:
                bins[b].append(i)
                loads[b] += lens[i]
                break
        else:
            bins.append([i])
            loads.append(lens[i])
    out = []
    for b in bins:
        b = sorted(b)
        ids, pos, msk, ret, cu = [], [], [], [], [0]
        for i in b:
            L = lens[i]
            ids.append(torch.tensor(samples[i].tokens[:L], dtype=torch.int64))
            pos.append(torch.arange(L, dtype=torch.int32))
            m, r = row_targets(samples[i], seq_len, gamma)
            msk.append(m)
            ret.append(r)
            cu.append(cu[-1] + L)
        out.append(CriticMicro(b, torch.cat(ids), torch.cat(pos), torch.tensor(cu, dtype=torch.int32),
                               max(lens[i] for i in b), torch.cat(msk), torch.cat(ret), [lens[i] for i in b]))
    return out


__all__ = ["CriticMicro", "TrajectorySample", "pack_micros", "row_targets", "sample_from_row", "samples_from_rows",
           "split_by_prompt"]
