"""Dynamic-batching planner: who trains which sample, in which micro-batch.

For one ``train_step`` over a global batch, a :class:`Plan` fixes

* the samples of each DP rank (equal counts, token-balanced),
* how a rank's samples split into mini-batches (one optimiser step each) and
  micro-batches (one forward/backward each), with each micro's row length,
* the *global* loss denominators of every mini-batch (documents and loss
  tokens summed over all ranks), so ranks need no extra collective.

It is a pure function of the sample lengths and :class:`PlannerConfig`; every
rank evaluates it on the same broadcast batch and gets the same answer.

Balancing rule (the one the reference planner uses, ``meshy/backend/titan/
plan.py:145-288``; kept because a mixed job must agree on it exactly):
samples are ranked by truncated length (longest first, lower index first on a
tie) and dealt back and forth over the bins (0, 1, .., n-1, n-1, .., 0, 0, ..)
-- first over DP ranks, then over a rank's mini-batches. Inside a mini-batch,
micro-batches are filled first-fit over the samples in the same order, with
the cost of a micro being rows x longest row (padded layout; a micro's first
sample is its longest) or the aligned token sum (packed layout). Ranks that
end up with fewer micros in a mini-batch are topped up with empty filler
micros so every rank runs the same number of forward passes.

This module's own structure: micro packing works on :class:`_OpenMicro`
accumulators, and the global denominators come from one per-(rank, mini)
table built once instead of being re-derived per rank.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Literal, Sequence

Layout = Literal["padded", "packed"]


def round_up(x: int, align: int) -> int:
    """Smallest multiple of ``align`` that is >= ``x``."""
    return ((x + align - 1) // align) * align


@dataclass(frozen=True)
class PlannerConfig:
    """Planner knobs. ``max_tokens_per_micro`` caps a micro's token cost; without it
    ``micro_batch_size`` caps its row count (padded layout only)."""

    layout: Layout
    mini_batch_size: int
    seq_len: int
    align: int
    max_tokens_per_micro: int | None = None
    micro_batch_size: int | None = None

    def __post_init__(self) -> None:
        problems = _config_problems(self)
        if problems:
            raise ValueError("invalid planner config: " + "; ".join(problems))


def _config_problems(c: PlannerConfig) -> list[str]:
    bad = []
    if c.layout not in ("padded", "packed"):
        bad.append(f"layout is {c.layout!r}, expected 'padded' or 'packed'")
    for name in ("mini_batch_size", "align", "seq_len"):
        if getattr(c, name) <= 0:
            bad.append(f"{name} = {getattr(c, name)} is not positive")
    if c.align > 0 and c.seq_len > 0 and c.seq_len % c.align:
        bad.append(f"seq_len {c.seq_len} is not a multiple of the row alignment {c.align}")
    for name in ("max_tokens_per_micro", "micro_batch_size"):
        v = getattr(c, name)
        if v is not None and v <= 0:
            bad.append(f"{name} = {v} is not positive")
    if c.max_tokens_per_micro is None:
        if c.layout == "packed":
            bad.append("the packed layout sizes micros by tokens: set max_tokens_per_micro")
        elif c.micro_batch_size is None:
            bad.append("set max_tokens_per_micro or micro_batch_size to bound a micro-batch")
    return bad


@dataclass(frozen=True)
class MicroPlan:
    """One forward/backward: batch positions of its samples, row length, and per-sample token counts.
    No samples means a filler micro (zero loss weight, keeps ranks in step)."""

    sample_idx: tuple[int, ...]
    seq_len: int
    doc_lens: tuple[int, ...]

    @property
    def is_filler(self) -> bool:
        return len(self.sample_idx) == 0

    @property
    def n_tokens(self) -> int:
        return sum(self.doc_lens)

    @property
    def n_rows(self) -> int:
        return len(self.sample_idx) or 1


@dataclass(frozen=True)
class MiniPlan:
    """One optimiser step of one rank, with the denominators of the whole DP group."""

    micros: tuple[MicroPlan, ...]
    n_docs_global: int
    n_tokens_global: int
    tokens_per_rank: tuple[int, ...]

    @property
    def n_docs_local(self) -> int:
        return sum(len(m.sample_idx) for m in self.micros)


@dataclass(frozen=True)
class Plan:
    """``per_rank[r]`` is rank r's mini-batches; ``local_indices[r]`` the batch indices it owns, in the
    order its micro ``sample_idx`` positions refer to."""

    per_rank: tuple[tuple[MiniPlan, ...], ...]
    local_indices: tuple[tuple[int, ...], ...]

    @property
    def dp_size(self) -> int:
        return len(self.per_rank)

    def local_samples(self, batch: Sequence, rank: int) -> list:
        return [batch[i] for i in self.local_indices[rank]]


def snake_deal(order: Sequence[int], n_bins: int) -> list[list[int]]:
    """Deal ``order`` over ``n_bins`` bins back and forth: 0..n-1, then n-1..0, and so on."""
    bins: list[list[int]] = [[] for _ in range(n_bins)]
    period = 2 * n_bins
    for k, item in enumerate(order):
        phase = k % period
        bins[phase if phase < n_bins else period - 1 - phase].append(item)
    return bins


def _longest_first(keys: Sequence[int], length_of) -> list[int]:
    return sorted(keys, key=lambda k: (-length_of(k), k))


class _OpenMicro:
    """A micro-batch being filled: its positions, their lengths, and its current extent (padded: the
    aligned first row; packed: the raw token sum)."""

    __slots__ = ("positions", "lengths", "extent")

    def __init__(self, pos: int, length: int, cfg: PlannerConfig):
        self.positions = [pos]
        self.lengths = [length]
        self.extent = round_up(length, cfg.align) if cfg.layout == "padded" else length

    def fits(self, length: int, cfg: PlannerConfig) -> bool:
        if cfg.max_tokens_per_micro is None:
            return len(self.positions) < cfg.micro_batch_size
        if cfg.layout == "padded":
            cost = (len(self.positions) + 1) * self.extent
        else:
            cost = round_up(self.extent + length, cfg.align)
        return cost <= cfg.max_tokens_per_micro

    def add(self, pos: int, length: int, cfg: PlannerConfig) -> None:
        self.positions.append(pos)
        self.lengths.append(length)
        if cfg.layout == "packed":
            self.extent += length

    def freeze(self, cfg: PlannerConfig) -> MicroPlan:
        row = self.extent if cfg.layout == "padded" else round_up(self.extent, cfg.align)
        return MicroPlan(tuple(self.positions), row, tuple(self.lengths))


def _pack_micros(positions: Sequence[int], lengths: Sequence[int], cfg: PlannerConfig) -> list[MicroPlan]:
    """First-fit of ``positions`` (longest first) into micros under the config's cost cap."""
    micros: list[_OpenMicro] = []
    for p in _longest_first(positions, lambda q: lengths[q]):
        home = next((m for m in micros if m.fits(lengths[p], cfg)), None)
        if home is None:
            micros.append(_OpenMicro(p, lengths[p], cfg))
        else:
            home.add(p, lengths[p], cfg)
    return [m.freeze(cfg) for m in micros]


def filler_micro(cfg: PlannerConfig) -> MicroPlan:
    """An empty micro of the minimum row length."""
    return MicroPlan((), cfg.align, ())


def build_plan(lengths: Sequence[int], loss_tokens: Sequence[int], dp_size: int, cfg: PlannerConfig) -> Plan:
    n = len(lengths)
    if n == 0 or len(loss_tokens) != n:
        raise ValueError(f"planner needs one loss-token count per sample and at least one sample "
                         f"(got {n} lengths, {len(loss_tokens)} loss-token counts)")
    if dp_size <= 0 or n % dp_size:
        raise ValueError(f"{n} samples cannot be split evenly over {dp_size} data-parallel ranks; choose a "
                         "rollout batch x group size that the DP degree divides")
    trunc = [min(int(L), cfg.seq_len) for L in lengths]
    owned = snake_deal(_longest_first(range(n), lambda i: trunc[i]), dp_size)
    per_rank_n = n // dp_size
    n_mini = math.ceil(per_rank_n / cfg.mini_batch_size)

    # rank r, mini i: the local positions of its samples, and its packed micros
    members: list[list[list[int]]] = []
    packed: list[list[list[MicroPlan]]] = []
    for r in range(dp_size):
        lens_r = [trunc[g] for g in owned[r]]
        groups = snake_deal(_longest_first(range(per_rank_n), lambda p: lens_r[p]), n_mini)
        members.append(groups)
        packed.append([_pack_micros(g, lens_r, cfg) for g in groups])

    # per (rank, mini): documents, loss tokens and truncated tokens -- summed over ranks below
    docs = [[len(members[r][i]) for i in range(n_mini)] for r in range(dp_size)]
    loss = [[sum(int(loss_tokens[owned[r][p]]) for p in members[r][i]) for i in range(n_mini)]
            for r in range(dp_size)]
    toks = [[sum(trunc[owned[r][p]] for p in members[r][i]) for i in range(n_mini)] for r in range(dp_size)]
    width = [max(len(packed[r][i]) for r in range(dp_size)) for i in range(n_mini)]

    filler = filler_micro(cfg)
    per_rank = []
    for r in range(dp_size):
        minis = []
        for i in range(n_mini):
            micros = tuple(packed[r][i]) + (filler,) * (width[i] - len(packed[r][i]))
            minis.append(MiniPlan(micros, sum(d[i] for d in docs), sum(x[i] for x in loss),
                                  tuple(t[i] for t in toks)))
        per_rank.append(tuple(minis))
    return Plan(tuple(per_rank), tuple(tuple(o) for o in owned))


def plan_stats(minis: Sequence[MiniPlan], layout: Layout) -> dict[str, float]:
    """Micro count, real tokens per micro, padding share of the forward tokens, and DP token imbalance
    (largest rank share over the mean) of a rank's mini-batches."""
    micros = [m for mini in minis for m in mini.micros]
    real = sum(m.n_tokens for m in micros)
    computed = sum(m.seq_len * (m.n_rows if layout == "padded" else 1) for m in micros)
    shares = [t for mini in minis for t in mini.tokens_per_rank]
    mean = sum(shares) / len(shares) if shares else 0.0
    return {
        "n_micro": float(len(micros)),
        "tokens_per_micro": real / max(1, len(micros)),
        "padding_ratio": 1.0 - real / max(1, computed),
        "dp_token_imbalance": float(max(shares) / mean) if mean > 0 else 1.0,
    }


def resolve_align(seq_bucket: int, divisor: int, seq_len: int) -> int:
    """Row-length granularity: the lcm of the padding bucket and the ``tp * cp * 2`` sequence divisor,
    capped at ``seq_len`` (which it must divide)."""
    align = min(math.lcm(max(1, seq_bucket), max(1, divisor)), seq_len)
    if seq_len % align:
        raise ValueError(f"row alignment {align} (lcm of bucket {seq_bucket} and divisor {divisor}) does not "
                         f"divide seq_len {seq_len}")
    return align


__all__ = [
    "Layout", "MicroPlan", "MiniPlan", "Plan", "PlannerConfig", "build_plan", "filler_micro",
    "plan_stats", "resolve_align", "round_up", "snake_deal",
]
