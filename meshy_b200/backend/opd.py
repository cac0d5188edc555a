"""Student side of Top-K on-policy distillation (reference ``meshy/backend/titan/opd.py:58-251``).

:class:`StudentTopKTrainer` is the PPO trainer with the loss replaced by the
forward KL to the teacher's Top-K distribution at every response position.
The teacher columns (``teacher_topk_ids`` / ``teacher_topk_logprobs``, one
``[L, K]`` array per row aligned with ``tokens``: row ``t`` is the teacher's
distribution over token ``t + 1``) are laid out on the micro-batch's packed
token stream exactly like the labels.  Aggregation matches the PPO loss:
per-sequence mean over response tokens then mean over the global number of
sequences (or the global token mean with ``calculate_per_token_loss``).  No
behaviour-policy snapshot is needed (no ratio).
"""

from __future__ import annotations

from typing import Any, Sequence

import torch
import torch.distributed as dist

from .plan import MiniPlan
from .topk_loss import forward_kl_topk, gather_logprobs
from .trainer import PPOTrainer

TEACHER_IDS, TEACHER_LPS = "teacher_topk_ids", "teacher_topk_logprobs"


def layout_teacher_topk(samples: Sequence[Any], micro, T: int, doc_starts: Sequence[int], device):
    k = None
    for idx in micro.sample_idx:
        k = torch.as_tensor(samples[idx][TEACHER_IDS]).shape[-1]
        break
    k = k or 1
    ids = torch.zeros(T, k, dtype=torch.long)
    lps = torch.zeros(T, k, dtype=torch.float32)
    for j, idx in enumerate(micro.sample_idx):
        L = micro.doc_lens[j]
        s = doc_starts[j]
        ti = torch.as_tensor(samples[idx][TEACHER_IDS])[:L]
        tl = torch.as_tensor(samples[idx][TEACHER_LPS])[:L]
        ids[s:s + ti.shape[0]] = ti.long()
        lps[s:s + tl.shape[0]] = tl.float()
    return ids.to(device, non_blocking=True), lps.to(device, non_blocking=True)


class StudentTopKTrainer(PPOTrainer):
    def __init__(self, *args, log_prob_min_clamp: float | None = -10.0, loss_max_clamp: float | None = 10.0, **kw):
        super().__init__(*args, **kw)
        self.log_prob_min_clamp = log_prob_min_clamp
        self.loss_max_clamp = loss_max_clamp

    @property
    def needs_behaviour_logprobs(self) -> bool:
        # the distillation loss has no PPO ratio
        return False

    def _doc_starts(self, b, micro) -> list[int]:
        if b.layout == "padded":
            return [j * micro.seq_len for j in range(len(micro.sample_idx))]
        out, off = [], 0
        for L in micro.doc_lens:
            out.append(off)
            off += L
        return out

    def _distill_loss(self, samples, micro, b, mini: MiniPlan):
        ids_t, lps_t = layout_teacher_topk(samples, micro, b.n_tokens, self._doc_starts(b, micro), self.device)
        k = ids_t.shape[-1]
        h = self.model.hidden(b.input_ids, b.positions, b.cu_seqlens, b.max_seqlen)
        ids = torch.cat([ids_t, b.labels.unsqueeze(-1)], -1)
        gathered = gather_logprobs(h, self.model.output_weight, ids)
        student, sampled = gathered[:, :k], gathered[:, k].detach()
        per_tok = forward_kl_topk(student, lps_t, log_prob_min_clamp=self.log_prob_min_clamp,
                                  loss_max_clamp=self.loss_max_clamp) * b.mask
        seg = per_tok.new_zeros(b.n_slots).index_add_(0, b.doc_ids, per_tok)
        n = b.n_docs
        if self.params.calculate_per_token_loss:
            loss = seg[:n].sum() / max(1, mini.n_tokens_global)
        else:
            loss = (seg[:n] / b.seg_count[:n].clamp(min=1)).sum() / max(1, mini.n_docs_global)
        with torch.no_grad():
            sums = {"loss": loss.detach().float(), "token_count": b.mask.sum().float(),
                    "student_mass_sum": (student.detach().exp().sum(-1) * b.mask).sum(),
                    "teacher_mass_sum": (lps_t.exp().sum(-1) * b.mask).sum()}
            if b.rollout_logprobs is not None:
                lr = (b.rollout_logprobs - sampled).clamp(-10.0, 10.0)
                sums["train_rollout_kl_sum"] = (torch.nan_to_num(lr.exp() - lr - 1.0) * b.mask).sum()
        return loss, sums

    def _run_mini_batch(self, samples, mini: MiniPlan, timer, old_lps=None):
        sums = None
        self.flat.zero_grad()
        for i, micro in enumerate(mini.micros):
            with timer.timer("train/pack_batch"):
                b = self._build(samples, micro, need_rollout_lp=True)
            with timer.timer("train/forward"):
                loss, mb = self._distill_loss(samples, micro, b, mini)
            with timer.timer("train/backward"):
                if micro.is_filler:
                    loss = loss * 0.0
                if i == len(mini.micros) - 1:
                    self.reducer.arm()
                loss.backward()
            sums = mb if sums is None else {k: sums[k] + v for k, v in mb.items()}
        self.flat.collect_cpu_grads()
        with timer.timer("train/grad_reduce"):
            self.reducer.finish()
        with timer.timer("train/optim_step"):
            gn = self.optimizer.step()
        keys = sorted(sums)
        st = torch.stack([sums[k].float().reshape(()) for k in keys]).to(self.device)
        if self.dp_group is not None and dist.is_initialized() and dist.get_world_size(self.dp_group) > 1:
            if dist.get_backend(self.dp_group) != "nccl":
                st = st.cpu()
            dist.all_reduce(st, group=self.dp_group)
        vals = dict(zip(keys, st.tolist()))
        tok = max(vals["token_count"], 1.0)
        out = {"train/distill_loss": vals["loss"], "train/student_topk_mass": vals["student_mass_sum"] / tok,
               "train/teacher_topk_mass": vals["teacher_mass_sum"] / tok}
        if "train_rollout_kl_sum" in vals:
            out["train_rollout_kl"] = vals["train_rollout_kl_sum"] / tok
        return out, gn


__all__ = ["StudentTopKTrainer", "TEACHER_IDS", "TEACHER_LPS", "layout_teacher_topk"]
