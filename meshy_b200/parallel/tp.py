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


def shard_model_tp(model, group) -> None:
    """Slice every block of ``model`` (a :class:`~meshy_b200.models.transformer.DecoderLM`) in place."""
    tp = dist.get_world_size(group)
    t = dist.get_rank(group)
    a = model.args
    if a.n_heads % tp or a.n_kv_heads % tp or (2 * a.ffn_dim) % (128 * tp):
        raise ValueError(f"TP={tp} must divide the heads ({a.n_heads}/{a.n_kv_heads}) and the 128-row gate/up "
                         f"blocks of 2F={2 * a.ffn_dim}")
    hd = a.head_dim
    hq, hkv = a.n_heads // tp, a.n_kv_heads // tp
    la = dataclasses.replace(a, n_heads=hq, n_kv_heads=hkv, ffn_dim=a.ffn_dim // tp)
    q_rows = torch.arange(t * hq * hd, (t + 1) * hq * hd)
    k_rows = a.n_heads * hd + torch.arange(t * hkv * hd, (t + 1) * hkv * hd)
    v_rows = (a.n_heads + a.n_kv_heads) * hd + torch.arange(t * hkv * hd, (t + 1) * hkv * hd)
    qkv_rows = torch.cat([q_rows, k_rows, v_rows])
    f_slice = slice(t * 2 * a.ffn_dim // tp, (t + 1) * 2 * a.ffn_dim // tp)
    w2_cols = torch.cat([torch.arange(b * 64, (b + 1) * 64) for b in range(f_slice.start // 128, f_slice.stop // 128)])
    with torch.no_grad():
        for blk in model.layers:
            dev = blk.wqkv.device
            blk.wqkv = nn.Parameter(blk.wqkv.index_select(0, qkv_rows.to(dev)).clone())
            if blk.bqkv is not None:
                blk.bqkv = nn.Parameter(blk.bqkv.index_select(0, qkv_rows.to(dev)).clone())
            blk.wo = nn.Parameter(blk.wo[:, t * hq * hd:(t + 1) * hq * hd].clone())
            if blk.moe is None:
                blk.w13 = nn.Parameter(blk.w13[f_slice].clone())
                blk.w2 = nn.Parameter(blk.w2.index_select(1, w2_cols.to(dev)).clone())
            blk.args = la
            blk.tp_group = group


__all__ = ["copy_to_tp", "reduce_from_tp", "shard_model_tp"]
