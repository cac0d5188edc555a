"""Process-group layout of a trainer replica: ``world = dp_replicate x dp_shard x cp x tp``.

Rank order (innermost fastest): ``tp``, then ``cp``, then ``dp_shard``, then
``dp_replicate`` -- the same nesting torchtitan's ``ParallelDims`` uses
(``TT:torchtitan/distributed/parallel_dims.py:84-200``), so a rank's
coordinates are a pure function of its global rank:

* ``batch`` group: ranks that see *different* samples (dp_replicate x dp_shard);
* ``cp`` group: ranks that split one sequence (head-tail chunks);
* ``tp`` group: ranks that split one layer's weights;
* ``loss`` group: ranks whose gradients are summed (batch x cp).

:func:`build_parallel_dims` creates every subgroup collectively (every rank
must call it, in the same order) and returns this rank's view.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch.distributed as dist


@dataclass
class ParallelDims:
    dp_replicate: int = 1
    dp_shard: int = 1
    cp: int = 1
    tp: int = 1
    rank: int = 0
    batch_group: object = None
    cp_group: object = None
    tp_group: object = None
    loss_group: object = None
    shard_group: object = None      # ranks that shard one replica's parameters (dp_shard x cp)
    replicate_group: object = None  # ranks that hold the same shard in different replicas

    @property
    def world(self) -> int:
        return self.dp_replicate * self.dp_shard * self.cp * self.tp

    @property
    def dp(self) -> int:
        return self.dp_replicate * self.dp_shard

    def coords(self, rank: int | None = None) -> dict[str, int]:
        r = self.rank if rank is None else rank
        tp = r % self.tp
        r //= self.tp
        cp = r % self.cp
        r //= self.cp
        return {"tp": tp, "cp": cp, "dp": r}

    @property
    def dp_rank(self) -> int:
        return self.coords()["dp"]

    @property
    def cp_rank(self) -> int:
        return self.coords()["cp"]

    @property
    def tp_rank(self) -> int:
        return self.coords()["tp"]


def _resolve(world: int, dp_replicate: int, dp_shard: int, cp: int, tp: int) -> tuple[int, int]:
    inner = cp * tp
    if dp_shard == -1 and dp_replicate == -1:
        raise ValueError("at most one of dp_shard / dp_replicate may be -1")
    if dp_shard == -1:
        dp_shard = world // (inner * dp_replicate)
    if dp_replicate == -1:
        dp_replicate = world // (inner * dp_shard)
    if dp_replicate * dp_shard * inner != world:
        raise ValueError(f"parallel degrees dp_replicate={dp_replicate} x dp_shard={dp_shard} x cp={cp} x tp={tp} "
                         f"!= world {world}")
    return dp_replicate, dp_shard


def build_parallel_dims(world: int, rank: int, *, dp_replicate: int = -1, dp_shard: int = 1, cp: int = 1,
                        tp: int = 1, backend: str | None = None) -> ParallelDims:
    dp_replicate, dp_shard = _resolve(world, dp_replicate, dp_shard, cp, tp)
    pd = ParallelDims(dp_replicate, dp_shard, cp, tp, rank)
    if world == 1 or not dist.is_initialized():
        return pd
    kw = {"backend": backend} if backend else {}
    dp = dp_replicate * dp_shard
    # every rank creates every group (new_group is collective), keeping its own
    for d in range(dp):
        for c in range(cp):
            ranks = [(d * cp + c) * tp + t for t in range(tp)]
            g = dist.new_group(ranks, **kw) if tp > 1 else None
            if rank in ranks:
                pd.tp_group = g
    for d in range(dp):
        for t in range(tp):
            ranks = [(d * cp + c) * tp + t for c in range(cp)]
            g = dist.new_group(ranks, **kw) if cp > 1 else None
            if rank in ranks:
                pd.cp_group = g
    for c in range(cp):
        for t in range(tp):
            ranks = [(d * cp + c) * tp + t for d in range(dp)]
            g = dist.new_group(ranks, **kw) if dp > 1 else None
            if rank in ranks:
                pd.batch_group = g
    for t in range(tp):
        ranks = [(d * cp + c) * tp + t for d in range(dp) for c in range(cp)]
        g = dist.new_group(ranks, **kw) if dp * cp > 1 else None
        if rank in ranks:
            pd.loss_group = g
    # replica-major DP index: d = rep * dp_shard + shard
    for rep in range(dp_replicate):
        for t in range(tp):
            ranks = [((rep * dp_shard + sh) * cp + c) * tp + t for sh in range(dp_shard) for c in range(cp)]
            g = dist.new_group(ranks, **kw) if dp_shard * cp > 1 else None
            if rank in ranks:
                pd.shard_group = g
    for sh in range(dp_shard):
        for c in range(cp):
            for t in range(tp):
                ranks = [((rep * dp_shard + sh) * cp + c) * tp + t for rep in range(dp_replicate)]
                g = dist.new_group(ranks, **kw) if dp_replicate > 1 else None
                if rank in ranks:
                    pd.replicate_group = g
    return pd


__all__ = ["ParallelDims", "build_parallel_dims"]
