"""GRPO/PPO clipped policy loss.

Semantics follow the reference (``meshy/backend/titan/trainer.py:705-848``):

* per-token ratio ``r = exp(new_lp - old_lp)``; asymmetric clip
  ``[1 - eps_low, 1 + eps_high]``; ``pg = -min(r A, clip(r) A)``;
* optional TIS (drop tokens whose ratio leaves ``[tis_min, tis_max]``) or
  IcePop (weight by ``exp(old_lp - rollout_lp)`` inside the band, 0 outside);
* optional positive-LM term ``-new_lp * w_doc``;
* sequence-mean aggregation (per-sample token mean, summed, divided by the
  mini-batch's global sample count) or token-mean (``/ n_tokens_global``);
* detached diagnostic sums (ratio, clip fraction, k1/k3 KL, ESS ...).

On CUDA the whole thing — forward terms, the analytic gradient with respect
to ``new_lp`` and every diagnostic sum — is one kernel
(``ppo_loss_fused`` in ``meshy_b200._C``); autograd only multiplies the saved
per-token gradient by the incoming scalar.  On CPU it is the plain PyTorch
expression below.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from ..ops.functional import native

SUM_KEYS = (
    "loss", "total_loss", "positive_lm_loss", "tis_ratio_sum", "ratio_sum", "clip_sum",
    "tis_masked_sum", "token_count", "ppo_kl_sum", "log_ratio_abs_sum", "ess_sum", "doc_count",
    "train_rollout_kl_sum", "train_rollout_logdiff_abs_sum", "entropy_sum",
)


@dataclass(frozen=True)
class LossConfig:
    eps_low: float = 0.2
    eps_high: float = 0.2
    use_tis: bool = False
    use_icepop: bool = False
    tis_min: float = 0.5
    tis_max: float = 5.0
    positive_lm_coef: float = 0.0
    per_token: bool = False
    train_old: bool = False  # old_lp comes from the trainer (train_rollout_kl uses old_lp)


def _denoms(batch, n_docs_global: int, n_tokens_global: int, per_token: bool):
    """Per-token normaliser ``1 / (count(doc) * n_docs_global)`` or ``1/n_tokens``."""
    if per_token:
        return torch.full_like(batch.mask, 1.0 / max(1, n_tokens_global))
    cnt = batch.seg_count.clamp(min=1.0)
    inv = 1.0 / (cnt * max(1, n_docs_global))
    inv = torch.cat([inv[: batch.n_docs], inv.new_zeros(1)])
    return inv[batch.doc_ids]


class _FusedPPO(torch.autograd.Function):
    @staticmethod
    def forward(ctx, new_lp, old_lp, adv_tok, mask, rollout_lp, inv_norm, pos_w_tok, entropy, doc_ids,
                n_slots, cfg):
        from ..ops._ext import ext

        C = ext()
        grad = torch.empty_like(new_lp)
        sums = torch.zeros(len(SUM_KEYS), dtype=torch.float32, device=new_lp.device)
        seg = torch.zeros(n_slots, 3, dtype=torch.float32, device=new_lp.device)
        C.ppo_loss_fused(new_lp, old_lp, adv_tok, mask, rollout_lp, inv_norm, pos_w_tok, entropy, doc_ids,
                         grad, sums, seg, cfg.eps_low, cfg.eps_high, int(cfg.use_tis), int(cfg.use_icepop),
                         cfg.tis_min, cfg.tis_max, cfg.positive_lm_coef, int(cfg.train_old))
        ctx.save_for_backward(grad)
        return sums[1].clone(), sums, seg

    @staticmethod
    def backward(ctx, gloss, gsums, gseg):
        (grad,) = ctx.saved_tensors
        return grad * gloss, None, None, None, None, None, None, None, None, None, None


def _ess_sums(seg_w, seg_w2, cnt, cp):
    """Effective-sample-size sums of one micro-batch.

    ``seg_w`` / ``seg_w2`` are this rank's per-sequence sums of the ratio and its square. Under context
    parallelism a sequence's tokens are spread over the ``cp`` ranks, so both are summed over the CP group
    first; every CP rank then holds the same per-sequence ESS, and the loss group's sum (DP x CP) counts each
    sequence ``cp`` times, which the division by the CP degree undoes (reference
    ``meshy/backend/titan/trainer.py:826-835``)."""
    deg = 1
    if cp is not None and cp.size > 1:
        both = cp.all_reduce_sum(torch.stack([seg_w, seg_w2]))
        seg_w, seg_w2, deg = both[0], both[1], cp.size
    ess = (seg_w * seg_w) / (cnt.clamp(min=1) * seg_w2.clamp(min=1e-8))
    live = (cnt > 0).to(ess.dtype)
    return (ess * live).sum() / deg, live.sum() / deg


def ppo_clip_loss(new_lp, old_lp, batch, n_docs_global: int, n_tokens_global: int, cfg: LossConfig,
                  entropy: torch.Tensor | None = None, cp=None):
    """Returns ``(loss, sums)``; ``sums`` is a dict of detached scalar tensors. ``cp`` is the context-parallel
    sharder (:class:`~meshy_b200.parallel.cp.CpSharder`) when sequences are split over a CP group."""
    mask = batch.mask
    adv = batch.advantages
    if batch.adv_per_token:
        adv_tok = adv
    else:
        adv_tok = torch.cat([adv, adv.new_zeros(1)])[batch.doc_ids]
    inv = _denoms(batch, n_docs_global, n_tokens_global, cfg.per_token)
    pos_w_tok = None
    if cfg.positive_lm_coef:
        if batch.positive_lm_weights is None:
            raise ValueError("Positive LM loss requires group weights")
        pos_w_tok = torch.cat([batch.positive_lm_weights, mask.new_zeros(1)])[batch.doc_ids]
    if cfg.use_icepop and batch.rollout_logprobs is None:
        raise ValueError("IcePop requires rollout log-probabilities")

    if native(new_lp):
        loss, sums_t, seg = _FusedPPO.apply(new_lp, old_lp, adv_tok, mask, batch.rollout_logprobs, inv,
                                            pos_w_tok, entropy, batch.doc_ids, batch.n_slots, cfg)
        # ESS needs the per-sequence sums of w and w^2 (seg[:, 0:2]) and counts
        sums = {k: sums_t[i] for i, k in enumerate(SUM_KEYS)}
        sums["ess_sum"], sums["doc_count"] = _ess_sums(seg[: batch.n_docs, 0], seg[: batch.n_docs, 1],
                                                       batch.seg_count[: batch.n_docs], cp)
        if batch.rollout_logprobs is None:
            sums.pop("train_rollout_kl_sum")
            sums.pop("train_rollout_logdiff_abs_sum")
        if entropy is None:
            sums.pop("entropy_sum")
        return loss, sums

    log_ratio = new_lp - old_lp
    ratio = log_ratio.exp()
    pg_un = ratio * adv_tok
    pg_cl = ratio.clamp(1 - cfg.eps_low, 1 + cfg.eps_high) * adv_tok
    pg = -torch.minimum(pg_un, pg_cl)
    tis_ratio = ratio.detach()
    if cfg.use_icepop:
        tis_ratio = (old_lp - batch.rollout_logprobs).detach().exp()
        tis_mask = (tis_ratio >= cfg.tis_min) & (tis_ratio <= cfg.tis_max)
        pg = torch.where(tis_mask, pg, 0) * torch.where(tis_mask, tis_ratio, 0)
    elif cfg.use_tis:
        tis_mask = (ratio >= cfg.tis_min) & (ratio <= cfg.tis_max)
        pg = torch.where(tis_mask, pg, torch.zeros_like(pg))
    else:
        tis_mask = torch.ones_like(ratio, dtype=torch.bool)
    pg = pg * mask
    pg_loss = (pg * inv).sum()
    positive_loss = (-new_lp * pos_w_tok * mask * inv).sum() if pos_w_tok is not None else pg_loss.new_zeros(())
    loss = pg_loss + cfg.positive_lm_coef * positive_loss
    with torch.no_grad():
        r, lr_ = ratio.detach(), log_ratio.detach()
        flat = batch.doc_ids
        seg_w = torch.zeros(batch.n_slots, dtype=r.dtype, device=r.device).index_add_(0, flat, r * mask)
        seg_w2 = torch.zeros(batch.n_slots, dtype=r.dtype, device=r.device).index_add_(0, flat, r * r * mask)
        n = batch.n_docs
        ess_sum, doc_count = _ess_sums(seg_w[:n], seg_w2[:n], batch.seg_count[:n], cp)
        sums = {
            "loss": pg_loss.detach(),
            "total_loss": loss.detach(),
            "positive_lm_loss": positive_loss.detach(),
            "tis_ratio_sum": (tis_ratio * mask).sum(),
            "ratio_sum": (r * mask).sum(),
            "clip_sum": (((r < 1 - cfg.eps_low) | (r > 1 + cfg.eps_high)).float() * mask).sum(),
            "tis_masked_sum": ((~tis_mask).float() * mask).sum(),
            "token_count": mask.sum(),
            "ppo_kl_sum": (-lr_ * mask).sum(),
            "log_ratio_abs_sum": (lr_.abs() * mask).sum(),
            "ess_sum": ess_sum,
            "doc_count": doc_count,
        }
        if batch.rollout_logprobs is not None:
            train_lp = old_lp if cfg.train_old else new_lp.detach()
            d = (batch.rollout_logprobs - train_lp).clamp(-10.0, 10.0)
            sums["train_rollout_kl_sum"] = (torch.nan_to_num(d.exp() - d - 1.0) * mask).sum()
            sums["train_rollout_logdiff_abs_sum"] = (
                torch.nan_to_num((batch.rollout_logprobs - train_lp).abs()) * mask).sum()
        if entropy is not None:
            sums["entropy_sum"] = (entropy.float() * mask).sum()
    return loss, sums


def reduce_sums(sums: dict[str, torch.Tensor], group=None) -> dict[str, float]:
    """Mini-batch metrics from per-rank sums (one all-reduce of a small vector)."""
    import torch.distributed as dist

    keys = list(sums)
    stacked = torch.stack([sums[k].float().reshape(()) for k in keys])
    if group is not None and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(stacked, group=group)
    v = dict(zip(keys, stacked.tolist()))
    tok = max(v["token_count"], 1.0)
    out = {
        "pg_loss": v["loss"],
        "ratio_mean": v["ratio_sum"] / tok,
        "clip_frac": v["clip_sum"] / tok,
        "tis_masked_frac": v["tis_masked_sum"] / tok,
        "ppo_kl": v["ppo_kl_sum"] / tok,
        "log_ratio_abs_mean": v["log_ratio_abs_sum"] / tok,
        "ess_ratio": v["ess_sum"] / max(v.get("doc_count", 0.0), 1.0),
        "tis_ratio_mean": v["tis_ratio_sum"] / tok,
        "positive_lm_loss": v["positive_lm_loss"],
        "total_loss": v["total_loss"],
    }
    if "train_rollout_kl_sum" in v:
        out["train_rollout_kl"] = v["train_rollout_kl_sum"] / tok
        out["train_rollout_logdiff_abs"] = v["train_rollout_logdiff_abs_sum"] / tok
    if "entropy_sum" in v:
        out["entropy"] = v["entropy_sum"] / tok
    return out


__all__ = ["LossConfig", "SUM_KEYS", "ppo_clip_loss", "reduce_sums"]
