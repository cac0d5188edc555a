"""Top-K on-policy distillation math (reference ``meshy/backend/titan/topk_loss.py:21-80``).

On the packed token stream ``h [T, D]`` (final-norm hidden states):

* :func:`teacher_topk` — the teacher's top-K next-token ids and their
  log-probabilities ``[T, K]``;
* :func:`gather_logprobs` — the student's log-probabilities of given ids
  ``[T, K]``, differentiable;
* :func:`forward_kl_topk` — per-position ``sum_k p_T(k) (log p_T(k) - log p_S(k))``
  over the teacher's K candidates, with the same clamps as the reference
  (both log-probs clamped from below, the per-token KL from above).

Both heads run the LM-head GEMM on ``chunk`` tokens at a time (the tcgen05
GEMM on CUDA), so the transient logits are bounded by ``[chunk, V]``; the
student's chunks are recomputed in backward (non-reentrant checkpoint) so
only one chunk of logits is alive at a time.
"""

from __future__ import annotations

import torch
from torch.utils.checkpoint import checkpoint

from ..ops import functional as Fx


@torch.no_grad()
def teacher_topk(h: torch.Tensor, w: torch.Tensor, k: int, *, chunk: int = 2048):
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


def gather_logprobs(h: torch.Tensor, w: torch.Tensor, ids: torch.Tensor, *, chunk: int = 2048) -> torch.Tensor:
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
