"""The decoder-only transformer used by the trainer, the critic and the teacher.

Parameter layout is chosen for the kernels, not copied from HF:

* ``wqkv [q_dim + 2 kv_dim, D]`` (+ ``bqkv``) — one GEMM for Q, K and V.
* ``w13 [2F, D]`` — gate and up rows interleaved in blocks of
  ``args.swiglu_block`` so the SwiGLU runs in the GEMM epilogue.
* ``w2 [D, F]``, ``wo [D, q_dim]``, ``lm_head [V, D]``.

The same tensors back the rollout engine when trainer and engine share a
process, so a weight update needs no re-layout.  :mod:`.hf` maps to and from
the HF checkpoint names.

The forward works on a *packed* token stream ``[T]`` with ``cu_seqlens`` (the
padded layout is the special case of one document per row), which is the
only layout the attention kernel needs.
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn
from torch.utils.checkpoint import checkpoint

from ..ops import functional as Fx
from .args import ModelArgs


class Block(nn.Module):
    def __init__(self, args: ModelArgs, layer_id: int):
        super().__init__()
        self.args = args
        self.layer_id = layer_id
        d = args.dim
        self.attn_norm = nn.Parameter(torch.ones(d))
        self.wqkv = nn.Parameter(torch.empty(args.qkv_dim, d))
        self.bqkv = nn.Parameter(torch.zeros(args.qkv_dim)) if args.qkv_bias else None
        if args.qk_norm:
            self.q_norm = nn.Parameter(torch.ones(args.head_dim))
            self.k_norm = nn.Parameter(torch.ones(args.head_dim))
        else:
            self.q_norm = self.k_norm = None
        self.wo = nn.Parameter(torch.empty(d, args.q_dim))
        self.mlp_norm = nn.Parameter(torch.ones(d))
        if args.moe is None:
            self.w13 = nn.Parameter(torch.empty(2 * args.ffn_dim, d))
            self.w2 = nn.Parameter(torch.empty(d, args.ffn_dim))
            self.moe = None
        else:
            from .moe import MoE

            self.moe = MoE(args)

    def reset_parameters(self, std: float = 0.02) -> None:
        depth_std = std / math.sqrt(2 * (self.layer_id + 1))
        nn.init.normal_(self.wqkv, std=std)
        nn.init.normal_(self.wo, std=depth_std)
        if self.moe is None:
            nn.init.normal_(self.w13, std=std)
            nn.init.normal_(self.w2, std=depth_std)
        else:
            self.moe.reset_parameters(std, depth_std)

    tp_group = None  # set by parallel.tp.shard_model_tp

    def forward(self, x, positions, cu_seqlens, max_seqlen):
        if self.tp_group is not None:
            return self._forward_tp(x, positions, cu_seqlens, max_seqlen)
        a = self.args
        T = x.shape[0]
        h = Fx.rmsnorm(x, self.attn_norm, a.norm_eps)
        qkv = Fx.linear(h, self.wqkv, self.bqkv)
        q, k, v = Fx.qkv_rope(qkv, positions, self.q_norm, self.k_norm, a.n_heads, a.n_kv_heads,
                              a.head_dim, a.rope_theta, a.norm_eps)
        o = Fx.flash_attn_varlen(q, k, v, cu_seqlens, max_seqlen)
        x = Fx.linear(o.reshape(T, a.q_dim), self.wo, residual=x)
        h = Fx.rmsnorm(x, self.mlp_norm, a.norm_eps)
        if self.moe is None:
            act = Fx.linear_swiglu(h, self.w13, a.swiglu_block)
            return Fx.linear(act, self.w2, residual=x)
        return x + self.moe(h)

    def _forward_tp(self, x, positions, cu_seqlens, max_seqlen):
        """Tensor-parallel block: this rank's heads / MLP slice, all-reduce after the row-parallel GEMMs."""
        from ..parallel.tp import copy_to_tp, reduce_from_tp

        a, g = self.args, self.tp_group
        T = x.shape[0]
        h = copy_to_tp(Fx.rmsnorm(x, self.attn_norm, a.norm_eps), g)
        qkv = Fx.linear(h, self.wqkv, self.bqkv)
        q, k, v = Fx.qkv_rope(qkv, positions, self.q_norm, self.k_norm, a.n_heads, a.n_kv_heads,
                              a.head_dim, a.rope_theta, a.norm_eps)
        o = Fx.flash_attn_varlen(q, k, v, cu_seqlens, max_seqlen)
        x = x + reduce_from_tp(Fx.linear(o.reshape(T, a.n_heads * a.head_dim), self.wo), g)
        h = copy_to_tp(Fx.rmsnorm(x, self.mlp_norm, a.norm_eps), g)
        act = Fx.linear_swiglu(h, self.w13, a.swiglu_block)
        return x + reduce_from_tp(Fx.linear(act, self.w2), g)


class DecoderLM(nn.Module):
    def __init__(self, args: ModelArgs, *, with_lm_head: bool = True):
        super().__init__()
        self.args = args
        self.embed = nn.Parameter(torch.empty(args.vocab_size, args.dim))
        self.layers = nn.ModuleList([Block(args, i) for i in range(args.n_layers)])
        self.norm = nn.Parameter(torch.ones(args.dim))
        if with_lm_head and not args.tie_embeddings:
            self.lm_head = nn.Parameter(torch.empty(args.vocab_size, args.dim))
        else:
            self.lm_head = None
        self.activation_checkpoint = False

    # ------------------------------------------------------------------
    def reset_parameters(self, seed: int = 0, std: float = 0.02) -> None:
        torch.manual_seed(seed)
        with torch.no_grad():
            nn.init.normal_(self.embed, std=std)
            for layer in self.layers:
                layer.reset_parameters(std)
            if self.lm_head is not None:
                nn.init.normal_(self.lm_head, std=1.0 / math.sqrt(self.args.dim))

    @property
    def output_weight(self) -> torch.Tensor:
        return self.lm_head if self.lm_head is not None else self.embed

    # ------------------------------------------------------------------
    def hidden(self, input_ids, positions, cu_seqlens, max_seqlen) -> torch.Tensor:
        """Final-norm hidden states ``[T, D]`` of a packed token stream."""
        # per-block hooks: the sharded-parameter engine (gathers / reduce-scatters) or the data-parallel
        # reducer (gradient all-reduce overlapped with the backward)
        fs = getattr(self, "fsdp", None) or getattr(self, "block_hooks", None)
        if fs is not None:
            fs.begin_forward()
        x = Fx.embedding(input_ids, self.embed)
        ckpt = self.activation_checkpoint and torch.is_grad_enabled()
        for i, layer in enumerate(self.layers):
            if fs is not None:
                x = fs.pre_block(i, x)
            if ckpt:
                x = checkpoint(layer, x, positions, cu_seqlens, max_seqlen, use_reentrant=False)
            else:
                x = layer(x, positions, cu_seqlens, max_seqlen)
            if fs is not None:
                x = fs.post_block(i, x)
        return Fx.rmsnorm(x, self.norm, self.args.norm_eps)

    def logprobs(self, input_ids, labels, positions, cu_seqlens, max_seqlen, *, with_entropy=False,
                 chunk: int = 4096):
        """Per-token ``log p(labels[t] | <= t)`` (fp32) and optional entropy."""
        h = self.hidden(input_ids, positions, cu_seqlens, max_seqlen)
        return Fx.lm_head_logprobs(h, self.output_weight, labels, with_entropy, chunk)

    def logits(self, input_ids, positions, cu_seqlens, max_seqlen) -> torch.Tensor:
        h = self.hidden(input_ids, positions, cu_seqlens, max_seqlen)
        return Fx.linear(h, self.output_weight)


def build_model(args: ModelArgs, *, seed: int = 0, device="cpu", dtype=torch.float32,
                with_lm_head: bool = True) -> DecoderLM:
    """Random-init model built directly on ``device`` (no host staging)."""
    with torch.device(device):
        m = DecoderLM(args, with_lm_head=with_lm_head)
        m.reset_parameters(seed)
    return m.to(dtype=dtype)


__all__ = ["Block", "DecoderLM", "build_model"]
