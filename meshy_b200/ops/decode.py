"""Inference-side ops of the rollout engine (no autograd).

* :func:`kv_write` — scatter this step's K/V rows into the paged cache.
* :func:`qkv_rope_to_cache` — QK-norm + RoPE with the K/V rows written
  straight into the paged cache (one kernel).
* :func:`linear_norm_prep` / :func:`linear_norm_scaled` — RMSNorm split across
  the residual GEMM that produces ``x`` (it writes ``bf16(g * x)`` and per-tile
  sums of squares) and the GEMM that consumes the norm (it scales its output
  rows by ``rstd``), so decode runs no separate normalisation kernels.
* :func:`paged_attention` — decode attention over the paged KV cache
  (split-KV flash-decode kernel on CUDA; GQA heads of one KV head share the
  K/V stream).
* :func:`sample` — fused LM head + softmax + categorical sample + log-prob.
  The CUDA kernel never writes logits: each CTA sweeps a vocab slice with
  tcgen05 tiles, keeps an online log-sum-exp and a Gumbel-max argmax per row,
  and a final pass merges the per-CTA partials.  Temperature-only sampling
  (every shipped recipe: temperature 1, top_p 1, top_k -1) takes this path;
  top-k / top-p write fp32 logits with the tcgen05 GEMM and filter and draw
  in one kernel per row (``_C.filtered_sample``), still without a host sync.
* :func:`decode_advance` — per-row bookkeeping after sampling (append token,
  bump lengths, recompute the next cache slot, finish flags), so a whole
  decode step can be replayed from a CUDA graph with no host work.
* :func:`sample_advance` — the decode step's tail in two kernels for up to 64
  rows: the LM head with the sampler in the epilogue of the small-M GEMM
  (vocabulary rows on the MMA's 128 lanes, tokens as its N; optionally on a
  prepared RMSNorm input, so the final norm runs no kernel of its own), then
  the partial merge fused with :func:`decode_advance` and ``step += 1``.
"""

from __future__ import annotations

import math

import torch

from . import reference as ref
from .functional import native


def kv_write(k, v, k_cache, v_cache, slot_mapping):
    """``k/v [B, Hkv, hd]`` → cache ``[n_pages, Hkv, page, hd]`` at ``slot_mapping [B]``."""
    from .checks import check_range

    check_range("KV-cache slots", slot_mapping, 0, k_cache.shape[0] * k_cache.shape[2])
    if native(k):
        from ._ext import ext

        ext().kv_write(k, v, k_cache, v_cache, slot_mapping)
        return
    page = k_cache.shape[2]
    pg = (slot_mapping // page).long()
    off = (slot_mapping % page).long()
    k_cache[pg, :, off] = k.to(k_cache.dtype)
    v_cache[pg, :, off] = v.to(v_cache.dtype)


def qkv_rope_to_cache(qkv, positions, q_norm, k_norm, n_heads, n_kv, hd, theta, eps, k_cache, v_cache,
                      slot_mapping, *, keep_kv: bool = False):
    """QK-norm + RoPE of a fused ``qkv [T, (Hq + 2 Hkv) hd]`` row block with K and V written straight
    into the paged cache at ``slot_mapping`` (one kernel instead of rope + scatter).

    Returns ``q [T, Hq, hd]`` and, with ``keep_kv`` (prefill needs them for attention), ``k, v``.
    """
    T = qkv.shape[0]
    if native(qkv):
        from ._ext import ext
        from .checks import check_range

        check_range("KV-cache slots", slot_mapping, 0, k_cache.shape[0] * k_cache.shape[2])
        q = torch.empty(T, n_heads, hd, dtype=qkv.dtype, device=qkv.device)
        k = torch.empty(T, n_kv, hd, dtype=qkv.dtype, device=qkv.device) if keep_kv else None
        v = torch.empty(T, n_kv, hd, dtype=qkv.dtype, device=qkv.device) if keep_kv else None
        ext().qkv_rope_cache(qkv, positions, q_norm, k_norm, q, k, v, k_cache, v_cache, slot_mapping, float(theta),
                             float(eps))
        return (q, k, v) if keep_kv else (q, None, None)
    from .functional import qkv_rope

    q, k, v = qkv_rope(qkv, positions, q_norm, k_norm, n_heads, n_kv, hd, theta, eps)
    kv_write(k, v, k_cache, v_cache, slot_mapping)
    return (q, k, v) if keep_kv else (q, None, None)


def linear_norm_prep(x, w, residual, g_next, xg, part):
    """``out = x W^T + residual`` that also prepares the next RMSNorm for :func:`linear_norm_scaled`:
    ``xg = bf16(out * g_next)`` and ``part[t, m]`` = sum of ``out[m]^2`` over output tile ``t``'s 128
    columns. Returns ``out``, or ``None`` when the fused small-M kernel does not apply (the caller
    then runs the unfused ops)."""
    if not native(x):
        return None
    from ._ext import ext

    out = torch.empty(x.shape[0], w.shape[0], dtype=x.dtype, device=x.device)
    if not ext().gemm_norm_prep(x, w, residual, out, xg[: x.shape[0]], g_next, part):
        return None
    return out


def linear_norm_scaled(xg, w, bias, part, d: int, eps: float, swiglu_block: int | None = None):
    """``epi(rstd * (xg W^T) + bias)`` with ``xg = bf16(g * x)`` and the row scale ``rstd`` rebuilt
    from the partial sums ``part`` written by :func:`linear_norm_prep` -- equal to
    ``linear(RMSNorm(x; g), W, bias)`` (SwiGLU epilogue with ``swiglu_block``). ``None`` when not
    applicable."""
    if not native(xg):
        return None
    from ._ext import ext

    n = w.shape[0]
    out = torch.empty(xg.shape[0], n // 2 if swiglu_block else n, dtype=xg.dtype, device=xg.device)
    epi = 1 if swiglu_block else 0
    if not ext().gemm_norm_scaled(xg, w, out, bias, part, (d + 127) // 128, float(d), float(eps), epi,
                                  int(swiglu_block or 0)):
        return None
    return out


def qkv_rope_fused(x, w, bias, positions, q_norm, k_norm, n_heads, n_kv, theta, eps, k_cache, v_cache, slot_mapping,
                   part=None, d: int = 0):
    """Decode QKV projection whose epilogue applies bias, (QK-norm), RoPE and writes K/V into the paged
    cache: returns ``q [T, Hq, 128]``, or ``None`` when the fused kernel does not apply. ``part``:
    ``x`` is a prepared RMSNorm input (see :func:`linear_norm_prep`) of model dim ``d``."""
    if not native(x) or w.shape[0] != (n_heads + 2 * n_kv) * 128 or k_cache.shape[-1] != 128:
        return None
    from ._ext import ext
    from .checks import check_range

    check_range("KV-cache slots", slot_mapping, 0, k_cache.shape[0] * k_cache.shape[2])
    T = x.shape[0]
    q = torch.empty(T, n_heads, 128, dtype=x.dtype, device=x.device)
    ok = ext().gemm_qkv_rope(x, w, bias, part, (d + 127) // 128 if part is not None else 0, float(d), float(eps),
                             positions, q_norm, k_norm, q, k_cache, v_cache, slot_mapping, float(theta), n_heads,
                             n_kv)
    return q if ok else None


def paged_attention(q, k_cache, v_cache, block_table, seq_lens, scale=None, workspace=None, decode_step=False):
    """Decode attention of ``q [B, Hq, hd]`` over each row's paged K/V. ``decode_step``: the op just
    before wrote only each row's newest K/V row (its position ``seq_lens - 1``) and neither the block
    table nor the lengths, so the kernel may load the older pages before that op has finished."""
    from .checks import check_paged

    check_paged("paged attention", block_table, seq_lens, k_cache.shape[0], k_cache.shape[2])
    scale = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    if native(q):
        from ._ext import ext

        out = torch.empty_like(q)
        ext().paged_attention(q, k_cache, v_cache, block_table, seq_lens, out, float(scale), workspace,
                              bool(decode_step))
        return out
    if q.is_cuda:
        return _library_paged_decode(q, k_cache, v_cache, block_table, seq_lens, scale)
    return ref.attention_decode_paged(q, k_cache, v_cache, block_table, seq_lens, scale)


def _library_paged_decode(q, k_cache, v_cache, block_table, seq_lens, scale):
    """Comparison baseline only: FlashAttention-2's paged KV-cache kernel (``flash_attn_with_kvcache``),
    the library kernel an SGLang/vLLM-class engine runs. It reads the cache through the block table with
    device-side lengths, so a decode step stays graph-capturable. It needs pages of a multiple of 256
    tokens; the cache ``[n_pages, Hkv, page, hd]`` is handed over as the strided view
    ``[n_pages, page, Hkv, hd]``."""
    from flash_attn import flash_attn_with_kvcache

    kc = k_cache.permute(0, 2, 1, 3)
    vc = v_cache.permute(0, 2, 1, 3)
    out = flash_attn_with_kvcache(q.unsqueeze(1), kc, vc, cache_seqlens=seq_lens, block_table=block_table,
                                  softmax_scale=scale, causal=True)
    return out.squeeze(1)


def sample(h, w, temperature: float, *, top_k: int = -1, top_p: float = 1.0, seed: int = 0,
           step: torch.Tensor | None = None, generator=None):
    """Returns ``(tokens int64 [B], logprobs fp32 [B])`` for hidden ``h [B, D]``.

    ``step`` is a device int64 counter folded into the Philox offset so a
    captured CUDA graph draws fresh noise every replay.
    """
    if native(h) and temperature > 0 and top_k <= 0 and top_p >= 1.0:
        from ._ext import ext

        B = h.shape[0]
        tok = torch.empty(B, dtype=torch.int64, device=h.device)
        lp = torch.empty(B, dtype=torch.float32, device=h.device)
        ext().lmhead_sample(h, w, tok, lp, float(temperature), int(seed), step)
        return tok, lp
    if native(h):  # top-k / top-p or greedy: fp32 logits from the tcgen05 GEMM, then the filtered sampler
        from ._ext import ext

        B, V = h.shape[0], w.shape[0]
        logits = torch.empty(B, V, dtype=torch.float32, device=h.device)
        ext().gemm(h.contiguous(), w, logits, False, False, None, None, None, 0, False, 0)
        tok = torch.empty(B, dtype=torch.int64, device=h.device)
        lp = torch.empty(B, dtype=torch.float32, device=h.device)
        ext().filtered_sample(logits, float(temperature), int(top_k), float(top_p), int(seed), step, tok, lp)
        return tok, lp
    if h.is_cuda and temperature > 0 and top_k <= 0 and top_p >= 1.0:
        return _library_sample(h, w, temperature)
    logits = h.float() @ w.float().t() if not h.is_cuda else torch.nn.functional.linear(h, w).float()
    return ref.sample_with_logprob(logits, temperature, generator=generator, top_k=top_k, top_p=top_p)


def _library_sample(h, w, temperature: float):
    """Comparison baseline only: cuBLAS logits, log-softmax, and an exponential-race draw
    (``argmax p / E`` with ``E ~ Exp(1)`` samples from ``p``), which stays graph-capturable."""
    logp = torch.log_softmax(torch.nn.functional.linear(h, w).float() / temperature, dim=-1)
    e = torch.empty_like(logp).exponential_()
    tok = (logp - e.log()).argmax(-1)
    return tok, logp.gather(-1, tok.unsqueeze(-1)).squeeze(-1)


def sample_advance(state: dict, h, w, temperature: float, *, seed: int, page_size: int, part=None, d: int = 0,
                   eps: float = 0.0) -> bool:
    """Sample the next token of every row from ``h [B, D]`` (temperature-only Gumbel-max sampling) and
    advance the rows (see :func:`decode_advance`), bumping ``state["step"]``. With ``part``, ``h`` is
    a prepared RMSNorm input ``bf16(g * x)`` of model dim ``d`` (see :func:`linear_norm_prep`). Returns
    False, having done nothing, when the fused kernels do not apply (no CUDA, > 64 rows, T <= 0)."""
    if not native(h) or not temperature > 0 or h.shape[0] > 64:
        return False
    from ._ext import ext

    st = state
    return bool(ext().decode_sample_advance(
        h, w, part, (d + 127) // 128 if part is not None else 0, float(d), float(eps), float(temperature), int(seed),
        st["step"], st["tok_in"], st["pos"], st["seq_lens"], st["gen"], st["max_new"], st["done"], st["slot"],
        st["block_table"], st["req"], st["out_tok"], st["out_lp"], st["eos"], int(page_size)))


def decode_advance(state: dict, tok, lp, page_size: int):
    """Append sampled tokens and advance per-row decode state (in place).

    ``state`` holds device tensors: ``tok_in [B]``, ``pos [B]``, ``seq_lens [B]``,
    ``gen [B]``, ``max_new [B]``, ``done [B]``, ``slot [B]``, ``block_table``,
    ``req [B]`` (output slot of the row), ``out_tok [R, L]``, ``out_lp [R, L]``,
    ``eos [n_eos]``.
    """
    if native(tok):
        from ._ext import ext

        ext().decode_advance(tok, lp, state["tok_in"], state["pos"], state["seq_lens"], state["gen"],
                             state["max_new"], state["done"], state["slot"], state["block_table"],
                             state["req"], state["out_tok"], state["out_lp"], state["eos"], int(page_size))
        return
    if tok.is_cuda:
        _advance_masked(state, tok, lp, page_size)
        return
    live = state["done"] == 0
    rows = torch.nonzero(live).flatten()
    if rows.numel() == 0:
        return
    r = state["req"][rows].long()
    g = state["gen"][rows].long()
    state["out_tok"][r, g] = tok[rows]
    state["out_lp"][r, g] = lp[rows]
    state["gen"][rows] += 1
    state["tok_in"][rows] = tok[rows]
    fin = state["gen"][rows] >= state["max_new"][rows]
    if state["eos"].numel():
        fin |= (tok[rows].unsqueeze(-1) == state["eos"].unsqueeze(0)).any(-1)
    state["done"][rows] = fin.to(state["done"].dtype)
    state["pos"][rows] += 1
    state["seq_lens"][rows] += 1
    p = state["pos"][rows].long()
    pg = state["block_table"][rows, p // page_size].long()
    state["slot"][rows] = pg * page_size + p % page_size


def _advance_masked(st: dict, tok, lp, page_size: int) -> None:
    """:func:`decode_advance` in torch ops with no host synchronisation (comparison baseline on CUDA, so
    its decode step can be graph-captured): every row is updated and finished rows keep their values."""
    B = tok.shape[0]
    live = st["done"][:B] == 0
    # rows that are not live write into the spare last output row, so they never collide with a live row
    trash = st["out_tok"].shape[0] - 1
    r = torch.where(live, st["req"][:B].long(), trash)
    g = torch.where(live, st["gen"][:B].long().clamp(max=st["out_tok"].shape[1] - 1), 0)
    st["out_tok"][r, g] = tok
    st["out_lp"][r, g] = lp.to(st["out_lp"].dtype)
    inc = live.to(st["gen"].dtype)
    st["gen"][:B] += inc
    st["tok_in"][:B] = torch.where(live, tok.to(st["tok_in"].dtype), st["tok_in"][:B])
    fin = st["gen"][:B] >= st["max_new"][:B]
    if st["eos"].numel():
        fin |= (tok.unsqueeze(-1) == st["eos"].unsqueeze(0)).any(-1)
    st["done"][:B] = torch.where(live, fin.to(st["done"].dtype), st["done"][:B])
    st["pos"][:B] += inc.to(st["pos"].dtype)
    st["seq_lens"][:B] += inc.to(st["seq_lens"].dtype)
    p = st["pos"][:B].long()
    pi = (p // page_size).clamp(max=st["block_table"].shape[1] - 1)
    pg = st["block_table"][:B].gather(1, pi.unsqueeze(1)).squeeze(1).long()
    st["slot"][:B] = torch.where(live, (pg * page_size + p % page_size).to(st["slot"].dtype), st["slot"][:B])


__all__ = ["decode_advance", "kv_write", "linear_norm_prep", "linear_norm_scaled", "paged_attention",
           "qkv_rope_fused", "qkv_rope_to_cache", "sample", "sample_advance"]
