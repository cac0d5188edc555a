"""Top-K on-policy distillation math (reference ``meshy/backend/titan/topk_loss.py:21-80``).

On the packed token stream ``h [T, D]`` (final-norm hidden states):

* :func:`teacher_topk` — the teacher's top-K next-token ids and their
  log-probabilities ``[T, K]``;
* :func:`gather_logprobs` — the student's log-probabilities of given ids
  ``[T, K]``, differentiable;
* :func:`forward_kl_topk` — per-position ``sum_k p_T(k) (log p_T(k) - log p_S(k))``
  over the teacher's K candidates, with the same clamps as the reference
  (both log-probs clamped from below, the per-token KL from above).

On CUDA both heads are native kernels:

* teacher: the tcgen05 GEMM writes one ``[chunk, V]`` fp32 block of logits and
  ``topk_logprobs`` (csrc/kernels/topk.cu) selects the K largest per row exactly
  (radix select), sorts them and subtracts the row's log-sum-exp, all in one
  kernel; the reference runs ``torch.topk`` and ``logsumexp`` on the same block;
* student: no logits are written in the forward. The LM-head GEMM's log-sum-exp
  epilogue gives ``lse`` per row and ``gather_logprobs`` takes the K dot
  products ``h_t . w[id]``; the backward forms ``dz = -G p`` in the GEMM
  epilogue (``G`` = the row's summed upstream gradient), adds the K one-hot
  terms with ``scatter_add_rows`` and feeds ``dz`` chunk by chunk to the dgrad
  and wgrad GEMMs.

The PyTorch path (CPU, and the library baseline) runs the GEMM on ``chunk``
tokens at a time and recomputes the student's chunks in backward
(non-reentrant checkpoint), so only one chunk of logits is alive at a time.
"""

from __future__ import annotations

import torch
from torch.utils.checkpoint import checkpoint

from ..ops import functional as Fx
from ..ops._ext import ext


_EPI_STORE, _EPI_NONE = 0, 0


@torch.no_grad()
def teacher_topk(h: torch.Tensor, w: torch.Tensor, k: int, *, chunk: int = 2048):
    if Fx.native(h):
        C = ext()
        T, V = h.shape[0], w.shape[0]
        ids = torch.empty(T, k, dtype=torch.long, device=h.device)
        lps = torch.empty(T, k, dtype=torch.float32, device=h.device)
        z = torch.empty(min(chunk, max(T, 1)), V, dtype=torch.float32, device=h.device)
        for s in range(0, T, chunk):
            e = min(T, s + chunk)
            zc = z[: e - s]
            C.gemm(h[s:e], w, zc, False, False, None, None, None, _EPI_STORE, False, 0)
            C.topk_logprobs(zc, k, ids[s:e], lps[s:e], None)
        return ids, lps
    ids, lps = [], []
    for s in range(0, h.shape[0], chunk):
        z = Fx.linear(h[s:s + chunk], w).float()
        top = z.topk(k, dim=-1)
        ids.append(top.indices)
        lps.append(top.values - torch.logsumexp(z, dim=-1, keepdim=True))
        del z
    return torch.cat(ids), torch.cat(lps)


def _chunk_gather(h: torch.Tensor, w: torch.Tensor, ids: torch.Tensor) -> torch.Tensor:
    z = Fx.linear(h, w).float()
    return z.gather(-1, ids) - torch.logsumexp(z, dim=-1, keepdim=True)


class _GatherLogprobs(torch.autograd.Function):
    """``log softmax(h W^T)[t, ids[t, k]]`` without [T, V] logits in the forward (see the module docstring)."""

    @staticmethod
    def forward(ctx, h, w, ids, chunk):
        C = ext()
        T = h.shape[0]
        lse = torch.empty(T, dtype=torch.float32, device=h.device)
        lp0 = torch.empty(T, dtype=torch.float32, device=h.device)
        C.lmhead_logprob_fwd(h, w, ids[:, 0].contiguous(), lp0, lse, None)
        lp = torch.empty(ids.shape, dtype=torch.float32, device=h.device)
        C.gather_logprobs(h, w, ids, lse, lp)
        ctx.save_for_backward(h, w, ids, lse)
        ctx.chunk = chunk
        return lp

    @staticmethod
    def backward(ctx, g):
        C = ext()
        h, w, ids, lse = ctx.saved_tensors
        T = h.shape[0]
        V = w.shape[0]
        g = g.float().contiguous()
        G = g.sum(-1).contiguous()
        none = torch.full((T,), -1, dtype=torch.long, device=h.device)
        gh = torch.empty_like(h)
        mg = getattr(w, "main_grad", None)
        gw32 = mg if mg is not None else torch.zeros(w.shape, dtype=torch.float32, device=w.device)
        chunk = max(128, min(ctx.chunk, T))
        dz = torch.empty(min(chunk, T), V, dtype=h.dtype, device=h.device)
        for s in range(0, T, chunk):
            e = min(T, s + chunk)
            dzc = dz[: e - s]
            C.lmhead_dlogits(h[s:e], w, none[s:e], lse[s:e], G[s:e], dzc)  # -G p
            C.scatter_add_rows(dzc, ids[s:e], g[s:e])                      # + sum_k g_k onehot(id_k)
            C.gemm(dzc, w, gh[s:e], False, True, None, None, None, _EPI_NONE, False, 0)
            C.gemm(dzc, h[s:e], gw32, True, True, None, None, None, _EPI_NONE, True, 0)
        gw = None if mg is not None else gw32.to(w.dtype)
        return gh, gw, None, None


def gather_logprobs(h: torch.Tensor, w: torch.Tensor, ids: torch.Tensor, *, chunk: int = 2048) -> torch.Tensor:
    if Fx.native(h):
        return _GatherLogprobs.apply(h.contiguous(), w, ids.long().contiguous(), chunk)
    recompute = torch.is_grad_enabled() and (h.requires_grad or w.requires_grad)
    out = []
    for s in range(0, h.shape[0], chunk):
        args = (h[s:s + chunk], w, ids[s:s + chunk].long())
        out.append(checkpoint(_chunk_gather, *args, use_reentrant=False) if recompute else _chunk_gather(*args))
    return torch.cat(out)


def forward_kl_topk(student_lp: torch.Tensor, teacher_lp: torch.Tensor, *, log_prob_min_clamp: float | None = None,
                    loss_max_clamp: float | None = None) -> torch.Tensor:
    log_s = student_lp.float()
    log_t = teacher_lp.float()
    if log_prob_min_clamp is not None:
        log_s = log_s.clamp_min(log_prob_min_clamp)
        log_t = log_t.clamp_min(log_prob_min_clamp)
    kl = (log_t.exp() * (log_t - log_s)).sum(-1)
    if loss_max_clamp is not None:
        kl = kl.clamp(min=-loss_max_clamp, max=loss_max_clamp)
    return kl


__all__ = ["forward_kl_topk", "gather_logprobs", "teacher_topk"]
