"""This package's parameter layout <-> torchtitan's fully qualified names (the reference trainer's DCP keys).

The reference trains torchtitan models and saves them with torchtitan's checkpointer, so a reference
checkpoint names weights ``tok_embeddings.weight``, ``layers.{i}.attention.qkv_linear.wq.weight``,
``layers.{i}.feed_forward.w1.weight``, ``layers.{i}.moe.experts.w1`` ... (the FQN tables of torchtitan's
Qwen3 / Llama3 state-dict adapters, which the reference's Qwen2.5 and MiniCPM5 adapters extend). This
package fuses some of them (``wqkv``, the block-interleaved ``w13``), so one of its parameters maps to one
or several torchtitan tensors: :func:`titan_pieces` splits, :func:`join_pieces` fuses back. Both work on
any tensor laid out like the parameter -- the AdamW moments included, which is what lets an optimiser
state move between the two layouts.

Llama-family models (``llama3``, ``minicpm5``): torchtitan applies RoPE to interleaved (even, odd) pairs,
HF and this package to the two halves of each head, so ``wq`` / ``wk`` rows are permuted on the way
(the same permutation the reference's MiniCPM5 adapter applies).
"""

from __future__ import annotations

import torch

from ..ops.reference import interleave_w13, split_w13
from .args import ModelArgs

_LLAMA_ROPE = ("llama3", "minicpm5")


def _to_interleaved(w: torch.Tensor, n_heads: int) -> torch.Tensor:
    """Rows of each head from (first half, second half) order to interleaved (even, odd) pairs."""
    rows, cols = w.shape[0], w.shape[1:]
    half = rows // n_heads // 2
    return w.reshape(n_heads, 2, half, *cols).transpose(1, 2).reshape(rows, *cols)


def _from_interleaved(w: torch.Tensor, n_heads: int) -> torch.Tensor:
    rows, cols = w.shape[0], w.shape[1:]
    half = rows // n_heads // 2
    return w.reshape(n_heads, half, 2, *cols).transpose(1, 2).reshape(rows, *cols)


def _split_qkv(args: ModelArgs, t: torch.Tensor):
    q, kv = args.q_dim, args.kv_dim
    wq, wk, wv = t[:q], t[q:q + kv], t[q + kv:]
    if args.name in _LLAMA_ROPE:
        wq, wk = _to_interleaved(wq, args.n_heads), _to_interleaved(wk, args.n_kv_heads)
    return wq, wk, wv


def titan_pieces(args: ModelArgs, name: str, t: torch.Tensor) -> list[tuple[str, torch.Tensor]]:
    """torchtitan (FQN, tensor) pieces of this package's parameter ``name`` (or of a tensor shaped like it)."""
    if name == "embed":
        return [("tok_embeddings.weight", t)]
    if name == "norm":
        return [("norm.weight", t)]
    if name == "lm_head":
        return [("lm_head.weight", t)]
    if not name.startswith("layers."):
        return [(name, t)]
    _, i, rest = name.split(".", 2)
    p = f"layers.{i}."
    if rest == "wqkv":
        wq, wk, wv = _split_qkv(args, t)
        return [(p + "attention.qkv_linear.wq.weight", wq), (p + "attention.qkv_linear.wk.weight", wk),
                (p + "attention.qkv_linear.wv.weight", wv)]
    if rest == "bqkv":
        bq, bk, bv = _split_qkv(args, t)
        return [(p + "attention.qkv_linear.wq.bias", bq), (p + "attention.qkv_linear.wk.bias", bk),
                (p + "attention.qkv_linear.wv.bias", bv)]
    simple = {"q_norm": "attention.q_norm.weight", "k_norm": "attention.k_norm.weight", "wo": "attention.wo.weight",
              "attn_norm": "attention_norm.weight", "mlp_norm": "ffn_norm.weight", "w2": "feed_forward.w2.weight",
              "moe.router": "moe.router.gate.weight", "moe.w2": "moe.experts.w2"}
    if rest in simple:
        return [(p + simple[rest], t)]
    if rest == "w13":
        g, u = split_w13(t, args.swiglu_block)
        return [(p + "feed_forward.w1.weight", g), (p + "feed_forward.w3.weight", u)]
    if rest == "moe.w13":
        parts = [split_w13(t[e], args.swiglu_block) for e in range(t.shape[0])]
        return [(p + "moe.experts.w1", torch.stack([g for g, _ in parts])),
                (p + "moe.experts.w3", torch.stack([u for _, u in parts]))]
    return [(p + rest, t)]


def join_pieces(args: ModelArgs, name: str, pieces: list[torch.Tensor]) -> torch.Tensor:
    """Inverse of :func:`titan_pieces`: the tensors of its FQNs, in its order, back to this package's layout."""
    rest = name.split(".", 2)[2] if name.startswith("layers.") else name
    if rest in ("wqkv", "bqkv"):
        q, k, v = pieces
        if args.name in _LLAMA_ROPE:
            q, k = _from_interleaved(q, args.n_heads), _from_interleaved(k, args.n_kv_heads)
        return torch.cat([q, k, v], 0)
    if rest == "w13":
        return interleave_w13(pieces[0], pieces[1], args.swiglu_block)
    if rest == "moe.w13":
        g, u = pieces
        return torch.stack([interleave_w13(g[e], u[e], args.swiglu_block) for e in range(g.shape[0])])
    (only,) = pieces
    return only


def titan_names(args: ModelArgs, name: str, shape) -> list[tuple[str, tuple[int, ...]]]:
    """FQNs and shapes of the pieces of a parameter of ``shape`` (no data needed)."""
    return [(n, tuple(x.shape)) for n, x in titan_pieces(args, name, torch.empty(shape, device="meta"))]


__all__ = ["join_pieces", "titan_names", "titan_pieces"]
