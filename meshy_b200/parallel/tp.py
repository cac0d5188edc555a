"""Tensor parallelism of the decoder blocks (Megatron-style column / row split).

Reference: torchtitan's TP plan for the Qwen blocks (``model.parallelize(tp_mesh)``,
``TT:torchtitan/models/qwen3/parallelize.py:58-61``), reachable from the
reference's config through ``tp_degree``.  Per TP rank ``t`` of ``tp``:

* attention: the fused ``wqkv`` keeps this rank's ``Hq / tp`` query heads and
  ``Hkv / tp`` KV heads (column split; ``bqkv`` and the QK-norm follow), ``wo``
  keeps the matching input columns (row split);
* MLP: ``w13`` keeps a contiguous ``2F / tp`` slice of the block-interleaved
  gate/up rows (a whole number of 128-row gate/up blocks, so every gate row
  keeps its up row), ``w2`` the matching ``F / tp`` input columns;
* norms, embedding and LM head stay replicated.

The block input enters the column-parallel GEMMs through ``copy_to_tp``
(identity forward, gradient all-reduce backward) and the row-parallel
outputs leave through ``reduce_from_tp`` (all-reduce forward, identity
backward), after which the residual is added once.  Replicated parameters see
identical activations on every TP rank, so no TP gradient reduction is needed;
the DP reduction runs over the batch group as usual.  Collectives go through
NCCL (gloo on CPU); the GEMM -> all-reduce fusion over NVLink is the planned
replacement.
"""

from __future__ import annotations

import dataclasses

import torch
import torch.distributed as dist
import torch.nn as nn


class _CopyToTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return x

    @staticmethod
    def backward(ctx, g):
        g = g.contiguous().clone()
        dist.all_reduce(g, group=ctx.group)
        return g, None


class _ReduceFromTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        y = x.contiguous().clone()
        dist.all_reduce(y, group=group)
        return y

    @staticmethod
    def backward(ctx, g):
        return g, None


def copy_to_tp(x, group):
    return _CopyToTP.apply(x, group)


def reduce_from_tp(x, group):
    return _ReduceFromTP.apply(x, group)


def _check_divisible(a, tp: int) -> None:
    if a.n_heads % tp or a.n_kv_heads % tp or (2 * a.ffn_dim) % (128 * tp):
        raise ValueError(f"TP={tp} must divide the heads ({a.n_heads}/{a.n_kv_heads}) and the 128-row gate/up "
                         f"blocks of 2F={2 * a.ffn_dim}")


def local_args(a, tp: int):
    """The block arguments one of ``tp`` ranks sees (its share of the heads and of the FFN width)."""
    _check_divisible(a, tp)
    return dataclasses.replace(a, n_heads=a.n_heads // tp, n_kv_heads=a.n_kv_heads // tp, ffn_dim=a.ffn_dim // tp)


def tp_shard_param(name: str, full: torch.Tensor, a, tp: int, t: int, ep: bool = False) -> torch.Tensor:
    """Rank ``t``'s slice of the block parameter ``name`` (its last dotted component: ``wqkv``, ``bqkv``,
    ``wo``, ``w13``, ``w2``; anything else is replicated and returned as is) from the full tensor. With ``ep``
    the MoE experts (``...moe.w13`` / ``...moe.w2``) are split over the ranks by expert: rank ``t`` keeps
    experts ``[t E/tp, (t + 1) E/tp)``."""
    leaf = name.rsplit(".", 1)[-1]
    if ep and ".moe." in name and leaf in ("w13", "w2"):
        n = full.shape[0] // tp
        return full[t * n:(t + 1) * n]
    hd = a.head_dim
    hq, hkv = a.n_heads // tp, a.n_kv_heads // tp
    dev = full.device
    if leaf in ("wqkv", "bqkv"):
        q_rows = torch.arange(t * hq * hd, (t + 1) * hq * hd)
        k_rows = a.n_heads * hd + torch.arange(t * hkv * hd, (t + 1) * hkv * hd)
        v_rows = (a.n_heads + a.n_kv_heads) * hd + torch.arange(t * hkv * hd, (t + 1) * hkv * hd)
        return full.index_select(0, torch.cat([q_rows, k_rows, v_rows]).to(dev))
    if leaf == "wo":
        return full[:, t * hq * hd:(t + 1) * hq * hd]
    if leaf == "w13" and ".moe." not in name:
        return full[t * 2 * a.ffn_dim // tp:(t + 1) * 2 * a.ffn_dim // tp]
    if leaf == "w2" and ".moe." not in name:
        f0, f1 = t * 2 * a.ffn_dim // tp, (t + 1) * 2 * a.ffn_dim // tp
        cols = torch.cat([torch.arange(b * 64, (b + 1) * 64) for b in range(f0 // 128, f1 // 128)])
        return full.index_select(1, cols.to(dev))
    return full


def shard_model_tp(model, group, ep: bool = False) -> None:
    """Slice every block of ``model`` (a :class:`~meshy_b200.models.transformer.DecoderLM`) in place. With ``ep``
    (inference) each rank also keeps only its share of every MoE layer's experts; the MoE output is then summed
    over ``group`` (every rank holds every token)."""
    tp = dist.get_world_size(group)
    t = dist.get_rank(group)
    a = model.args
    la = local_args(a, tp)
    with torch.no_grad():
        for blk in model.layers:
            for leaf in ("wqkv", "bqkv", "wo"):
                w = getattr(blk, leaf)
                if w is not None:
                    setattr(blk, leaf, nn.Parameter(tp_shard_param(leaf, w, a, tp, t).clone()))
            if blk.moe is None:
                blk.w13 = nn.Parameter(tp_shard_param("w13", blk.w13, a, tp, t).clone())
                blk.w2 = nn.Parameter(tp_shard_param("w2", blk.w2, a, tp, t).clone())
            elif ep:
                moe = blk.moe
                if moe.n_experts % tp:
                    raise ValueError(f"EP={tp} must divide the {moe.n_experts} experts")
                moe.w13 = nn.Parameter(tp_shard_param(".moe.w13", moe.w13, a, tp, t, ep=True).clone())
                moe.w2 = nn.Parameter(tp_shard_param(".moe.w2", moe.w2, a, tp, t, ep=True).clone())
                moe.expert_offset = t * (moe.n_experts // tp)
                moe.ep_tokens_group = group
            blk.args = la
            blk.tp_group = group


__all__ = ["copy_to_tp", "local_args", "reduce_from_tp", "shard_model_tp", "tp_shard_param"]
