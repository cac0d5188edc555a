"""In-process colocated GRPO/PPO step: the rollout engine and the trainer share a GPU.

This is the B200 layout of the reference's JustRL recipe (``recipe/justrl.py``:
8 x TP1 inference replicas colocated with a DDP8 trainer, lock-step pacing)
without any process or network hop inside a rank:

1. the rank's :class:`~meshy_b200.rollout.RolloutEngine` generates
   ``group_size`` completions per prompt (paged KV, CUDA-graph decode);
2. rewards (a rule function) and group-normalised advantages
   (``grpo_advantage``, reference ``meshy/worker/rollout.py:88-97``);
3. the :class:`~meshy_b200.backend.trainer.PPOTrainer` recomputes behaviour
   log-probs, runs the PPO mini-batches with the DDP gradient reduction, and
   steps AdamW;
4. weight sync: the trainer's bf16 compute weights (what AdamW just wrote)
   are copied into the engine's bf16 weight buffer (same flat layout; one
   device copy, no disk, no gather).

Across ranks only the gradient reduction and the loss denominators travel.
The service-based path (launcher → TransferQueue → workers) drives the same
trainer and engine classes; this module is the shortest way to one step.
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Callable, Sequence

import torch
import torch.distributed as dist

from .advantage import grpo_advantage_values
from .backend.plan import MiniPlan, Plan, build_plan
from .backend.trainer import PPOTrainer
from .config import TrainerConfig, TrainerParamsConfig
from .rollout import RolloutEngine


@dataclass
class StepReport:
    metrics: dict
    n_samples: int
    n_tokens: int
    n_response_tokens: int
    times: dict = field(default_factory=dict)


def parity_reward(prompt: Sequence[int], response: Sequence[int]) -> float:
    """Rule reward used by the synthetic benchmark: 1 if the response id sum is even."""
    return 1.0 if (sum(response) % 2 == 0) else 0.0


class ColocatedGRPO:
    def __init__(
        self,
        trainer_config: TrainerConfig,
        trainer_params: TrainerParamsConfig,
        *,
        device: str | torch.device,
        group_size: int = 8,
        temperature: float = 1.0,
        dp_group=None,
        seed: int = 0,
        reward_fn: Callable[[Sequence[int], Sequence[int]], float] = parity_reward,
        engine_kwargs: dict | None = None,
        ignore_eos: bool = True,
        release_kv_for_training: bool = False,
    ):
        self.device = torch.device(device)
        # the engine's KV pages are idle while the trainer runs; releasing them (virtual addresses kept, so the
        # decode graphs stay valid) frees their memory for the trainer, but the release also empties the
        # allocator's cache, and the trainer's next forward re-allocates everything (measured slower: off)
        self.release_kv = release_kv_for_training
        self.trainer = PPOTrainer(trainer_config, trainer_params, device=self.device, dp_group=dp_group, seed=seed)
        ek = dict(engine_kwargs or {})
        self.engine = RolloutEngine(self.trainer.model_args, device=self.device, seed=seed + 1000 * self.rank,
                                    model=_engine_model(self.trainer), **ek)
        self.sync_weights()
        self.group_size = group_size
        self.temperature = temperature
        self.reward_fn = reward_fn
        self.ignore_eos = ignore_eos
        self.dp_group = dp_group
        self.version = 0

    @property
    def rank(self) -> int:
        return dist.get_rank() if dist.is_initialized() else 0

    # ------------------------------------------------------------------
    def sync_weights(self) -> float:
        """Trainer fp32 master → engine bf16 weights (device cast copy); returns ms."""
        if self.device.type == "cuda":
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            self.engine.update_weights_from_flat(self.trainer.flat.sync_source, version=getattr(self, "version", 0))
            e.record()
            e.synchronize()
            return s.elapsed_time(e)
        t0 = time.perf_counter()
        self.engine.update_weights_from_flat(self.trainer.flat.sync_source, version=getattr(self, "version", 0))
        return (time.perf_counter() - t0) * 1e3

    def rollout(self, prompts: Sequence[Sequence[int]], max_new_tokens: Sequence[int] | int):
        G = self.group_size
        flat_prompts = [p for p in prompts for _ in range(G)]
        if isinstance(max_new_tokens, int):
            max_new_tokens = [max_new_tokens] * len(flat_prompts)
        gens = self.engine.generate(flat_prompts, list(max_new_tokens), temperature=self.temperature,
                                    ignore_eos=self.ignore_eos)
        samples = []
        for i, g in enumerate(gens):
            r = self.reward_fn(g.prompt_ids, g.output_ids)
            tokens = torch.tensor(g.prompt_ids + g.output_ids, dtype=torch.long)
            mask = torch.zeros(len(tokens), dtype=torch.float32)
            mask[len(g.prompt_ids):] = 1.0
            lps = torch.zeros(len(tokens), dtype=torch.float32)
            lps[len(g.prompt_ids):] = torch.tensor(g.output_logprobs, dtype=torch.float32)
            samples.append({
                "tokens": tokens, "logprobs": lps, "mask_assistant": mask, "reward": torch.tensor(r),
                "weight_version": torch.tensor(g.weight_version), "truncated": torch.tensor(
                    int(g.finish_reason == "length")), "repetition": torch.tensor(0),
                "mixed_version": torch.tensor(0), "group": i // G,
            })
        for gi in range(len(prompts)):
            grp = samples[gi * G:(gi + 1) * G]
            for s, a in zip(grp, grpo_advantage_values([float(s["reward"]) for s in grp])):
                s["advantage"] = torch.tensor(a)
        return samples

    def plan_local(self, samples) -> tuple[list, Sequence[MiniPlan]]:
        """Plan this rank's samples; loss denominators are summed over the DP group."""
        t = self.trainer
        lengths, loss_tokens = t.sample_lengths(samples, t.config.seq_len)
        plan: Plan = build_plan(lengths, loss_tokens, 1, t.planner_config)
        minis = list(plan.per_rank[0])
        self.last_wait_s = 0.0
        if self.dp_group is not None and dist.is_initialized() and dist.get_world_size(self.dp_group) > 1:
            dev = self.device if dist.get_backend(self.dp_group) == "nccl" else torch.device("cpu")
            cnt = torch.tensor([[m.n_docs_global, m.n_tokens_global] for m in minis], dtype=torch.float64,
                               device=dev)
            # the step's first cross-rank collective: a rank whose rollout finished early waits here for the
            # slowest one (the all-reduce plus the read-back is host-synchronous, so this is device time)
            t_wait = time.perf_counter()
            dist.all_reduce(cnt, group=self.dp_group)
            cnt = cnt.cpu().long().tolist()
            self.last_wait_s = time.perf_counter() - t_wait
            minis = [MiniPlan(m.micros, c[0], c[1], m.tokens_per_rank) for m, c in zip(minis, cnt)]
        return plan.local_samples(samples, 0), minis

    def step(self, prompts: Sequence[Sequence[int]], max_new_tokens: Sequence[int] | int) -> StepReport:
        """One lock-step GRPO iteration on this rank (collective across the DP group)."""
        from .utils.timer import nvtx_range

        times = {}
        t0 = time.perf_counter()
        with nvtx_range("rl/rollout"):
            samples = self.rollout(prompts, max_new_tokens)
        times["rollout_s"] = time.perf_counter() - t0
        if self.release_kv:
            self.engine.release_memory(("kv_cache",))
        t1 = time.perf_counter()
        with nvtx_range("rl/train"):
            local, minis = self.plan_local(samples)
            metrics = self.trainer.train_step(local, plan=minis)
        times["train_s"] = time.perf_counter() - t1
        if self.release_kv:
            self.engine.resume_memory(("kv_cache",))
        times["wait_s"] = getattr(self, "last_wait_s", 0.0)
        times["optim_s"] = float(metrics.get("time/train/optim_step", 0.0)) + float(
            metrics.get("time/train/grad_reduce", 0.0))
        times["train_compute_s"] = times["train_s"] - times["wait_s"]
        self.version += 1
        with nvtx_range("rl/weight_sync"):
            times["weight_sync_ms"] = self.sync_weights()
        n_tok = sum(len(s["tokens"]) for s in samples)
        n_resp = sum(int(s["mask_assistant"].sum()) for s in samples)
        metrics["rollout/raw_reward_mean"] = sum(float(s["reward"]) for s in samples) / max(1, len(samples))
        return StepReport(metrics, len(samples), n_tok, n_resp, times)


def _engine_model(trainer: PPOTrainer):
    """A separate bf16 model object for the engine (its own weight buffer)."""
    from .models import build_model

    dt = torch.bfloat16 if trainer.device.type == "cuda" else torch.float32
    return build_model(trainer.model_args, seed=0, device=trainer.device, dtype=dt)


__all__ = ["ColocatedGRPO", "StepReport", "parity_reward"]
