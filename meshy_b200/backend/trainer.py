"""The PPO/GRPO trainer (replaces the reference's torchtitan ``TitanTrainer``).

One instance per rank.  Public surface mirrors the reference
(``meshy/backend/titan/trainer.py:854-1185``): ``plan_batch``,
``train_step(samples, plan=..., step_schedule=...)`` returning a metrics
dict, behaviour-policy recompute before the first optimiser step, GAE attach,
checkpoint save/load and HF export.

Inside, the B200 design:

* parameters, gradients and optimiser states are flat buffers
  (:mod:`.flat`); kernels accumulate weight gradients in fp32 directly;
* the data-parallel gradient reduction works on the flat gradient: on one
  node the fused NVLink optimiser step (:mod:`meshy_b200.parallel.symm`:
  reduce-scatter, norm, AdamW on the shard, all-gather) runs after the
  backward; otherwise per-block NCCL all-reduces start inside the last
  micro-batch's backward (:mod:`meshy_b200.parallel.ddp`); with sharded
  parameters (:mod:`meshy_b200.parallel.fsdp`) each block's gradient is
  reduce-scattered as its backward ends;
* the log-prob head is the fused LM-head kernel (no ``[T, V]`` logits), the
  loss is the fused PPO kernel, the step is one AdamW kernel that can also
  write the bf16 weights of a colocated rollout engine (weight sync).
"""

from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Any, Sequence

import torch
import torch.distributed as dist

from ..config import TrainerConfig, TrainerParamsConfig
from ..models import build_model, get_model_args
from ..utils.timer import TimerStats
from .batch import ADVANTAGE_TOKENS, Batch, build_micro_batch
from .flat import FlatAdamW, FlatParams, lr_lambda
from .loss import LossConfig, ppo_clip_loss, reduce_sums
from .plan import MiniPlan, Plan, PlannerConfig, build_plan, filler_micro, plan_stats, resolve_align


@dataclass
class StepTimes:
    old_logprobs: float = 0.0
    forward_backward: float = 0.0
    optimizer: float = 0.0


class PPOTrainer:
    def __init__(
        self,
        config: TrainerConfig,
        params: TrainerParamsConfig | None = None,
        *,
        device: str | torch.device = "cpu",
        dp_group=None,
        seed: int = 0,
        model=None,
        timer_enabled: bool = True,
        cp_group=None,
        loss_group=None,
        ep_group=None,
        tp_group=None,
        fsdp_group=None,
        replicate_group=None,
    ):
        self.config = config
        self.params = params or TrainerParamsConfig()
        self.device = torch.device(device)
        self.dp_group = dp_group
        # context parallelism: sequences split head-tail over cp_group; gradients and loss sums then
        # reduce over the loss group (DP x CP), the data split stays over DP
        self.cp = None
        if cp_group is not None and dist.is_initialized() and dist.get_world_size(cp_group) > 1:
            from ..parallel.cp import CpSharder

            self.cp = CpSharder(cp_group)
        self.loss_group = loss_group if loss_group is not None else dp_group
        self.model_args = get_model_args(config.model_name, config.model_flavor)
        cdt = torch.bfloat16 if (self.device.type == "cuda" and config.dtype == "bfloat16") else torch.float32
        self.compute_dtype = cdt
        if model is None:
            model = build_model(self.model_args, seed=seed, device=self.device, dtype=torch.float32)
        # expert parallelism: this rank keeps 1/ep of every MoE layer's experts (ep_group = the DP ranks
        # that split the experts); their gradients are never summed over that group
        self.tp_group = tp_group
        if tp_group is not None and dist.is_initialized() and dist.get_world_size(tp_group) > 1:
            from ..parallel.tp import shard_model_tp

            shard_model_tp(model, tp_group)
        self.ep_group = ep_group
        if ep_group is not None and dist.is_initialized() and dist.get_world_size(ep_group) > 1:
            from ..parallel.ep import shard_experts

            p = self.params
            # tokens of the largest micro-batch: the peer-memory exchange sizes its receive regions for it
            max_tokens = p.max_tokens_per_micro or config.seq_len * max(1, p.micro_batch_size or 1)
            shard_experts(model, ep_group, max_tokens=max_tokens)
        self.model = model
        self.model.activation_checkpoint = config.activation_checkpoint_mode == "full"
        # fully sharded parameters (FSDP over fsdp_group, HSDP with a replicate group on top)
        self.fsdp = fsdp_group is not None and dist.is_initialized()
        if self.fsdp:
            if self.ep_group is not None or (self.tp_group is not None and dist.get_world_size(self.tp_group) > 1):
                raise ValueError("sharded parameters combine with data and context parallelism only")
            from ..parallel.fsdp import ShardedFlat

            self.flat = ShardedFlat(self.model, fsdp_group, compute_dtype=cdt, device=self.device,
                                    replicate_group=replicate_group)
            self.model.fsdp = self.flat
        else:
            self.flat = FlatParams(self.model, compute_dtype=cdt, device=self.device)
        if cdt != torch.float32:
            torch.cuda.empty_cache()
        self.optimizer = FlatAdamW(self.flat, lr=config.lr, betas=(config.beta1, config.beta2), eps=config.eps,
                                   weight_decay=config.weight_decay, max_norm=config.max_norm)
        self.step = 0
        self.timer_enabled = timer_enabled
        p = self.params
        self.loss_cfg = LossConfig(
            eps_low=p.ppo_clip_eps_low, eps_high=p.ppo_clip_eps_high, use_tis=p.use_tis, use_icepop=p.use_icepop,
            tis_min=p.tis_ratio_min, tis_max=p.tis_ratio_max, positive_lm_coef=p.positive_lm_loss_coef,
            per_token=p.calculate_per_token_loss, train_old=p.old_logprobs_source == "train",
        )
        self.batch_layout = p.batch_layout
        divisor = max(1, config.tp_degree * config.cp_degree * (2 if config.cp_degree > 1 else 1))
        self.align = resolve_align(p.seq_bucket if p.batch_layout == "padded" else 64, divisor, config.seq_len)
        self.planner_config = PlannerConfig(
            layout=p.batch_layout, mini_batch_size=p.mini_batch_size, seq_len=config.seq_len, align=self.align,
            max_tokens_per_micro=p.max_tokens_per_micro,
            micro_batch_size=None if p.max_tokens_per_micro is not None else p.micro_batch_size,
        )
        from ..parallel.ddp import GradReducer

        expert_slots = [(sl.offset, sl.numel) for sl in self.flat.slots
                        if ".moe.w13" in sl.name or ".moe.w2" in sl.name] if self.ep_group is not None else []
        if self.fsdp:
            # the gradient shards are reduced inside backward; replicas of a shard sum theirs here
            rg = replicate_group if (replicate_group is not None and dist.get_world_size(replicate_group) > 1) \
                else None
            self.reducer = GradReducer(self.flat, rg, backend=None if rg is not None else "none")
        else:
            self.reducer = GradReducer(self.flat, self.loss_group, skip=expert_slots)
        # under TP the per-head QK-norm gains are replicated but each rank's gradient covers only its
        # heads: those slots are summed over the TP group before the DP reduction
        self.tp_partial = [(sl.offset, sl.numel) for sl in self.flat.slots
                           if sl.name.endswith(".q_norm") or sl.name.endswith(".k_norm")] \
            if (self.tp_group is not None and dist.is_initialized() and dist.get_world_size(self.tp_group) > 1) else []
        self.fused_dp = False
        if self._use_fused_dp():
            # DDP gradient reduction + AdamW as one NVLink pipeline (reduce-scatter, norm, shard update,
            # all-gather by P2P stores); the reducer has nothing left to do
            from ..parallel.symm import FusedDPAdamW

            self.optimizer = FusedDPAdamW(self.flat, self.loss_group, lr=config.lr, betas=(config.beta1, config.beta2),
                                          eps=config.eps, weight_decay=config.weight_decay, max_norm=config.max_norm)
            # heap-resident buffers stay mapped while the trainer is offloaded (the fp32 master stays only
            # when it is the replicated weight buffer, i.e. without a bf16 compute copy)
            self.flat.resident = ("grad", "compute") if self.flat.separate_compute else ("master", "grad", "compute")
            self.reducer.backend = "none"
            self.fused_dp = True
        if not self.fsdp and self.reducer.overlapping:
            self.model.block_hooks = self.reducer  # per-block all-reduce during the last micro's backward
        self.h2d_bytes = 0

    def _use_fused_dp(self) -> bool:
        import os

        if os.environ.get("MESHY_DP_FUSED", "auto") == "0" or self.device.type != "cuda" or self.fsdp:
            return False
        from ..ops.functional import native

        if not native(self.flat.grad):  # library comparison baseline: NCCL all-reduce + PyTorch AdamW
            return False
        if self.ep_group is not None:  # expert slices differ per rank: keep the range-aware reducer
            return False
        g = self.loss_group
        if g is None or not dist.is_initialized() or dist.get_world_size(g) < 2:
            return False
        if dist.get_backend(g) != "nccl":
            return False
        from ..parallel.symm import SymmetricHeap

        return SymmetricHeap.supported(g)

    # ------------------------------------------------------------------ planning
    @property
    def dp_size(self) -> int:
        if self.dp_group is None or not dist.is_initialized():
            return 1
        return dist.get_world_size(self.dp_group)

    @property
    def dp_rank(self) -> int:
        if self.dp_group is None or not dist.is_initialized():
            return 0
        return dist.get_rank(self.dp_group)

    @staticmethod
    def sample_lengths(samples: Sequence[Any], seq_len: int) -> tuple[list[int], list[int]]:
        lengths, loss_tokens = [], []
        for td in samples:
            n = int(len(td["tokens"]))
            L = min(n, seq_len)
            lengths.append(n)
            m = td["mask_assistant"]
            loss_tokens.append(int((torch.as_tensor(m[1:L]) > 0).sum()) if L > 1 else 0)
        return lengths, loss_tokens

    def plan_batch(self, samples: Sequence[Any], dp_size: int | None = None) -> Plan:
        lengths, loss_tokens = self.sample_lengths(samples, self.config.seq_len)
        return build_plan(lengths, loss_tokens, dp_size or self.dp_size, self.planner_config)

    # ------------------------------------------------------------------ forward
    def _build(self, samples, micro, need_rollout_lp=True) -> Batch:
        b = build_micro_batch(samples, micro, layout=self.batch_layout, device=self.device,
                              need_rollout_lp=need_rollout_lp, sharder=self.cp)
        self.h2d_bytes += b.h2d_bytes
        return b

    def forward_batch(self, b: Batch, with_entropy: bool = False):
        if self.cp is not None and "cp" in b.extra:
            from ..parallel.cp import cp_attention

            with cp_attention(self.cp, b.extra["cp"]):
                return self.model.logprobs(b.input_ids, b.labels, b.positions, b.cu_seqlens, b.max_seqlen,
                                           with_entropy=with_entropy, chunk=self.params.logprob_chunk_size * 4)
        return self.model.logprobs(b.input_ids, b.labels, b.positions, b.cu_seqlens, b.max_seqlen,
                                   with_entropy=with_entropy, chunk=self.params.logprob_chunk_size * 4)

    @torch.no_grad()
    def compute_old_logprobs(self, samples, mini: MiniPlan) -> list[torch.Tensor]:
        out = []
        for micro in mini.micros:
            b = self._build(samples, micro, need_rollout_lp=False)
            lp, _ = self.forward_batch(b)
            out.append(lp)
        return out

    @property
    def needs_behaviour_logprobs(self) -> bool:
        return True

    # ------------------------------------------------------------------ GAE
    def attach_gae_advantages(self, samples: Sequence[Any]) -> dict[str, float]:
        from .gae import attach_gae

        p = self.params
        return attach_gae(samples, self.config.seq_len, gamma=p.gae_gamma, alpha=p.gae_alpha, lam=p.gae_lambda,
                          normalize=p.normalize_advantages, group=self.dp_group)

    # ------------------------------------------------------------------ step
    def train_step(self, samples: list[Any], *, plan: Sequence[MiniPlan] | None = None,
                   step_schedule: bool = True) -> dict[str, float]:
        timer = TimerStats(enabled=self.timer_enabled)
        if plan is None:
            with timer.timer("train/plan"):
                full = self.plan_batch(samples, 1)
                samples = full.local_samples(samples, 0)
                plan = full.per_rank[0]
        if self.fsdp:
            plan = self._equalize_micros(plan)
        gae_metrics: dict[str, float] = {}
        if self.params.enable_gae:
            with timer.timer("train/gae"):
                gae_metrics = self.attach_gae_advantages(samples)

        old_per_mini: list[list[torch.Tensor] | None] = [None] * len(plan)
        if self.params.old_logprobs_source == "train" and self.needs_behaviour_logprobs:
            with timer.timer("train/old_logprobs", sync=True):
                old_per_mini = [self.compute_old_logprobs(samples, mini) for mini in plan]

        all_metrics, norms = [], []
        for i, mini in enumerate(plan):
            m, gn = self._run_mini_batch(samples, mini, timer, old_per_mini[i])
            old_per_mini[i] = None
            all_metrics.append(m)
            norms.append(gn)
        if step_schedule:
            self.step += 1
            c = self.config
            self.optimizer.lr = self.optimizer.base_lr * lr_lambda(
                self.step, warmup=c.warmup_steps, total=c.steps, decay_ratio=c.lr_decay_ratio,
                decay_type=c.lr_decay_type, min_factor=c.lr_min_factor)
        result: dict[str, float] = {}
        for key in all_metrics[0]:
            result[key] = sum(mm[key] for mm in all_metrics) / len(all_metrics)
        nv = [float(g) for g in norms]
        result["grad_norm"] = sum(nv) / len(nv)
        result["grad_norm_max"] = max(nv)
        result["grad_norm_last"] = nv[-1]
        result["step"] = self.step
        result["lr"] = self.optimizer.lr
        result.update(timer.pop_metrics(prefix="time/"))
        for k, v in plan_stats(plan, self.batch_layout).items():
            result[f"train/{k}"] = float(v)
        result["num_mini_batches"] = float(len(plan))
        result.update(gae_metrics)
        return result

    def _run_mini_batch(self, samples, mini: MiniPlan, timer: TimerStats, old_lps=None):
        if old_lps is None:
            old_lps = [None] * len(mini.micros)
        sums = None
        self.flat.zero_grad()
        n_micro = len(mini.micros)
        for i, (micro, old_lp) in enumerate(zip(mini.micros, old_lps)):
            with timer.timer("train/pack_batch"):
                b = self._build(samples, micro)
            if old_lp is None:
                if b.rollout_logprobs is None:
                    raise ValueError("old_logprobs_source='rollout' but the batch has no rollout log-probs")
                old_lp = b.rollout_logprobs
            with timer.timer("train/forward"):
                new_lp, ent = self.forward_batch(b, with_entropy=self.params.log_entropy)
                loss, mb_sums = ppo_clip_loss(new_lp, old_lp, b, mini.n_docs_global, mini.n_tokens_global,
                                              self.loss_cfg, entropy=ent, cp=self.cp)
            with timer.timer("train/backward"):
                if micro.is_filler:
                    loss = loss * 0.0
                last = i == n_micro - 1
                if last:
                    self.reducer.arm()
                loss.backward()
                self.flat.collect_cpu_grads()  # PyTorch paths only: fold .grad into the fp32 buffer
            sums = mb_sums if sums is None else {k: sums[k] + v for k, v in mb_sums.items()}
        with timer.timer("train/grad_reduce"):
            self.reducer.finish()  # first: it waits for the reductions the backward started
            for off, n in self.tp_partial:
                dist.all_reduce(self.flat.grad[off:off + n], group=self.tp_group)
        with timer.timer("train/optim_step"):
            gn = self.optimizer.step(self._ep_grad_norm() if self.reducer.skip else None)
        return reduce_sums(sums, self.loss_group), gn

    def _equalize_micros(self, plan: Sequence[MiniPlan]) -> list[MiniPlan]:
        """Sharded parameters gather and reduce inside every micro-batch, so every rank of the shard group
        must run the same number of them: pad each mini-batch with empty filler micros up to the group's
        largest count (a rank-local plan, as the lock-step loop builds, can differ from rank to rank)."""
        g = self.flat.group
        dev = self.device if dist.get_backend(g) == "nccl" else torch.device("cpu")
        n = torch.tensor([len(plan), -len(plan)], dtype=torch.int64, device=dev)
        dist.all_reduce(n, op=dist.ReduceOp.MAX, group=g)
        if int(n[0]) != -int(n[1]):
            raise ValueError(f"ranks of the shard group planned {-int(n[1])} to {int(n[0])} mini-batches; sharded "
                             "parameters need the same number on every rank")
        counts = torch.tensor([len(m.micros) for m in plan] or [0], dtype=torch.int64, device=dev)
        dist.all_reduce(counts, op=dist.ReduceOp.MAX, group=g)
        filler = filler_micro(self.planner_config)
        out = []
        for m, c in zip(plan, counts.tolist()):
            if c > len(m.micros):
                m = MiniPlan(tuple(m.micros) + (filler,) * (c - len(m.micros)), m.n_docs_global, m.n_tokens_global,
                             m.tokens_per_rank)
            out.append(m)
        return out

    def _ep_grad_norm(self) -> torch.Tensor:
        """Global gradient norm under expert parallelism: the dense part is replicated (counted once),
        every rank's experts are its own (their squared norms are summed over the EP group), so all ranks
        clip with the same coefficient."""
        g = self.flat.grad
        exp_sq = torch.zeros((), dtype=torch.float32, device=g.device)
        for off, n in self.reducer.skip:
            exp_sq = exp_sq + g[off:off + n].float().pow(2).sum()
        total_sq = g.float().pow(2).sum()
        dense_sq = total_sq - exp_sq
        if dist.is_initialized() and dist.get_world_size(self.ep_group) > 1:
            t = exp_sq.reshape(1).clone()
            if dist.get_backend(self.ep_group) != "nccl":
                t = t.cpu()
            dist.all_reduce(t, group=self.ep_group)
            exp_sq = t.to(g.device).reshape(())
        return (dense_sq + exp_sq).sqrt()

    # ------------------------------------------------------------------ weights
    def named_weights(self):
        """``(name, compute-dtype tensor)`` in the flat layout order."""
        for s, p in zip(self.flat.slots, self.flat.params):
            yield s.name, p

    def state_dict(self) -> dict[str, Any]:
        return {"step": self.step, "model": self.flat.state_dict(), "optim": self.optimizer.state_dict()}

    def load_state_dict(self, sd: dict[str, Any]) -> None:
        self.step = int(sd["step"])
        self.flat.load_state_dict(sd["model"])
        self.optimizer.load_state_dict(sd["optim"])

    def save_checkpoint(self, path: str, step: int | None = None) -> None:
        from .checkpoint import save_trainer_state

        save_trainer_state(self, path, self.step if step is None else step)

    def load_checkpoint(self, path: str) -> None:
        from .checkpoint import load_trainer_state

        load_trainer_state(self, path)

    def export_hf(self, output_dir: str) -> str:
        from ..models.hf import save_hf_checkpoint

        # the replicated compute weights: valid on every rank, whatever shards the fp32 master
        return save_hf_checkpoint(self.model_args, self.flat.state_dict(source="compute"), output_dir)

    def offload_to_cpu(self) -> None:
        """Colocation hand-off: move every flat buffer to pinned host memory."""
        from .offload import offload

        offload(self)

    def restore_to_gpu(self) -> None:
        from .offload import restore

        restore(self)


__all__ = ["PPOTrainer", "StepTimes"]
