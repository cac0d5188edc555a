"""Dynamic-batching planner.

A plan answers, for one ``train_step`` over a global batch: which samples
each DP rank owns (equal counts, balanced tokens), how a rank's samples form
mini-batches (one optimiser step each) and micro-batches (one forward each),
the row length of every micro-batch, and the *global* loss denominators of
each mini-batch.

The planner is a pure function of the sample lengths and the config, so every
rank plans the same broadcast batch without further communication.  The
steps are the reference's (``meshy/backend/titan/plan.py:145-288``) because
ranks of a mixed job must agree on them exactly:

1. sort by truncated length (desc, index tiebreak) and deal boustrophedon
   ("snake") into DP ranks;
2. per rank, snake-deal again into mini-batches;
3. per mini-batch, first-fit-decreasing packing under ``max_tokens_per_micro``
   (padded: rows × first-row length; packed: aligned token sum);
4. pad every rank to the same micro count per mini-batch with zero-weight
   filler micros, and attach ``n_docs_global`` / ``n_tokens_global``.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Literal, Sequence

Layout = Literal["padded", "packed"]


@dataclass(frozen=True)
class PlannerConfig:
    layout: Layout
    mini_batch_size: int
    seq_len: int
    align: int
    max_tokens_per_micro: int | None = None
    micro_batch_size: int | None = None

    def __post_init__(self) -> None:
        if self.layout not in ("padded", "packed"):
            raise ValueError(f"unknown layout {self.layout!r}")
        if self.mini_batch_size <= 0:
            raise ValueError("mini_batch_size must be positive")
        if self.align <= 0 or self.seq_len <= 0:
            raise ValueError("align and seq_len must be positive")
        if self.seq_len % self.align:
            raise ValueError(f"seq_len ({self.seq_len}) must be a multiple of align ({self.align})")
        if self.max_tokens_per_micro is not None and self.max_tokens_per_micro <= 0:
            raise ValueError("max_tokens_per_micro must be positive")
        if self.micro_batch_size is not None and self.micro_batch_size <= 0:
            raise ValueError("micro_batch_size must be positive")
        if self.max_tokens_per_micro is None and self.micro_batch_size is None:
            raise ValueError("either max_tokens_per_micro or micro_batch_size must be set")
        if self.layout == "packed" and self.max_tokens_per_micro is None:
            raise ValueError("packed layout requires max_tokens_per_micro")


@dataclass(frozen=True)
class MicroPlan:
    """One forward/backward. Empty ``sample_idx`` marks a filler micro."""

    sample_idx: tuple[int, ...]
    seq_len: int
    doc_lens: tuple[int, ...]

    @property
    def is_filler(self) -> bool:
        return not self.sample_idx

    @property
    def n_tokens(self) -> int:
        return sum(self.doc_lens)

    @property
    def n_rows(self) -> int:
        return max(1, len(self.sample_idx))


@dataclass(frozen=True)
class MiniPlan:
    micros: tuple[MicroPlan, ...]
    n_docs_global: int
    n_tokens_global: int
    tokens_per_rank: tuple[int, ...]

    @property
    def n_docs_local(self) -> int:
        return sum(len(m.sample_idx) for m in self.micros)


@dataclass(frozen=True)
class Plan:
    per_rank: tuple[tuple[MiniPlan, ...], ...]
    local_indices: tuple[tuple[int, ...], ...]

    @property
    def dp_size(self) -> int:
        return len(self.per_rank)

    def local_samples(self, batch: Sequence, rank: int) -> list:
        return [batch[i] for i in self.local_indices[rank]]


def round_up(x: int, align: int) -> int:
    return -(-x // align) * align


def snake_deal(order: Sequence[int], n_bins: int) -> list[list[int]]:
    """Deal ``order`` boustrophedon into ``n_bins`` lists."""
    bins: list[list[int]] = [[] for _ in range(n_bins)]
    for k, item in enumerate(order):
        rnd, pos = divmod(k, n_bins)
        bins[pos if rnd % 2 == 0 else n_bins - 1 - pos].append(item)
    return bins


def _pack_micros(positions: Sequence[int], lengths: Sequence[int], cfg: PlannerConfig) -> list[MicroPlan]:
    order = sorted(positions, key=lambda p: (-lengths[p], p))
    budget = cfg.max_tokens_per_micro
    row_cap = cfg.micro_batch_size if budget is None else None
    open_micros: list[tuple[list[int], list[int], list[int]]] = []  # (pos, lens, [extent])
    for p in order:
        L = lengths[p]
        for pos, lens, ext in open_micros:
            if row_cap is not None and len(pos) >= row_cap:
                continue
            if budget is not None:
                if cfg.layout == "padded":
                    cost = (len(pos) + 1) * ext[0]
                else:
                    cost = round_up(ext[0] + L, cfg.align)
                if cost > budget:
                    continue
            pos.append(p)
            lens.append(L)
            if cfg.layout == "packed":
                ext[0] += L
            break
        else:
            open_micros.append(([p], [L], [round_up(L, cfg.align) if cfg.layout == "padded" else L]))
    out = []
    for pos, lens, ext in open_micros:
        seq = ext[0] if cfg.layout == "padded" else round_up(ext[0], cfg.align)
        out.append(MicroPlan(tuple(pos), seq, tuple(lens)))
    return out


def filler_micro(cfg: PlannerConfig) -> MicroPlan:
    return MicroPlan((), cfg.align, ())


def build_plan(lengths: Sequence[int], loss_tokens: Sequence[int], dp_size: int, cfg: PlannerConfig) -> Plan:
    n = len(lengths)
    if n == 0:
        raise ValueError("cannot plan an empty batch")
    if len(loss_tokens) != n:
        raise ValueError("lengths and loss_tokens must have the same size")
    if dp_size <= 0 or n % dp_size:
        raise ValueError(
            f"batch size {n} is not divisible by DP size {dp_size}; make rollout batch x group size "
            "a multiple of the data-parallel degree"
        )
    trunc = [min(int(L), cfg.seq_len) for L in lengths]
    rank_samples = snake_deal(sorted(range(n), key=lambda i: (-trunc[i], i)), dp_size)
    n_local = n // dp_size
    n_mini = -(-n_local // cfg.mini_batch_size)

    minis_by_rank, members_by_rank = [], []
    for r in range(dp_size):
        local_len = [trunc[g] for g in rank_samples[r]]
        members = snake_deal(sorted(range(n_local), key=lambda p: (-local_len[p], p)), n_mini)
        members_by_rank.append(members)
        minis_by_rank.append([_pack_micros(m, local_len, cfg) for m in members])

    per_rank = []
    for r in range(dp_size):
        minis = []
        for i in range(n_mini):
            n_micro = max(len(minis_by_rank[q][i]) for q in range(dp_size))
            micros = list(minis_by_rank[r][i]) + [filler_micro(cfg)] * (n_micro - len(minis_by_rank[r][i]))
            n_docs = sum(len(members_by_rank[q][i]) for q in range(dp_size))
            n_tok = 0
            tpr = []
            for q in range(dp_size):
                gl = [rank_samples[q][p] for p in members_by_rank[q][i]]
                n_tok += sum(int(loss_tokens[g]) for g in gl)
                tpr.append(sum(trunc[g] for g in gl))
            minis.append(MiniPlan(tuple(micros), n_docs, n_tok, tuple(tpr)))
        per_rank.append(tuple(minis))
    return Plan(tuple(per_rank), tuple(tuple(s) for s in rank_samples))


def plan_stats(minis: Sequence[MiniPlan], layout: Layout) -> dict[str, float]:
    n_micro = real = fwd = 0
    for mini in minis:
        for m in mini.micros:
            n_micro += 1
            real += m.n_tokens
            fwd += (m.n_rows if layout == "padded" else 1) * m.seq_len
    tpr = [t for mini in minis for t in mini.tokens_per_rank]
    mean = sum(tpr) / max(1, len(tpr))
    return {
        "n_micro": float(n_micro),
        "tokens_per_micro": real / max(1, n_micro),
        "padding_ratio": 1.0 - real / max(1, fwd),
        "dp_token_imbalance": float(max(tpr) / mean) if mean > 0 else 1.0,
    }


def resolve_align(seq_bucket: int, divisor: int, seq_len: int) -> int:
    """Row-length granularity: lcm of the bucket and the ``tp*cp*2`` divisor."""
    align = math.lcm(max(1, seq_bucket), max(1, divisor))
    if align >= seq_len:
        align = seq_len
    if seq_len % align:
        raise ValueError(
            f"seq_len ({seq_len}) must be a multiple of the sequence alignment ({align} = "
            f"lcm(seq_bucket={seq_bucket}, divisor={divisor}))"
        )
    return align


__all__ = [
    "Layout", "MicroPlan", "MiniPlan", "Plan", "PlannerConfig", "build_plan", "filler_micro",
    "plan_stats", "resolve_align", "round_up", "snake_deal",
]
