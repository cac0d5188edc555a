"""Critic replica engine (reference ``meshy/engine/critic.py:26-601``).

``score_and_train(samples, publish, global_step)`` on rank 0 broadcasts the
window; every rank takes its token-balanced share (snake deal over lengths,
the planner's DP split), runs one accumulated value step
(:class:`~meshy_b200.backend.critic.trainer.CriticTrainer`), and rank 0
gathers the pre-update values of every row.  With ``publish`` the engine
returns per-row ``values`` (the trainer computes VAPO-GAE from them) or, in
``advantage`` mode, the per-sequence GAE advantage it computes itself.
Global checkpoints (trainer state + a sidecar) go to the run's state store;
offload/restore move the flat buffers for colocation hand-offs.
"""

from __future__ import annotations

import logging
import os
from typing import Any

import torch
import torch.distributed as dist

from ..backend.critic.data import samples_from_rows, split_by_prompt
from ..backend.critic.metrics import StreamingGauges, critic_diagnostics
from ..backend.critic.trainer import CriticTrainer
from ..backend.plan import snake_deal
from ..config import GlobalCheckpointConfig
from ..models import get_model_args
from .spmd import SpmdEngine

log = logging.getLogger(__name__)


class CriticSpmdEngine(SpmdEngine):
    def __init__(self, config, *, service_name: str, runtime=None, **kw):
        super().__init__(**kw)
        self.cfg = config
        self.service_name = service_name
        self.runtime = runtime
        self.checkpoint = GlobalCheckpointConfig.coerce(getattr(config, "checkpoint", None))
        self.trainer: CriticTrainer | None = None
        self.gauges = StreamingGauges()
        self.windows = 0
        self.weight_version = 0

    def setup(self) -> None:
        super().setup()
        c = self.cfg
        tc = c.trainer_config
        args = get_model_args(tc.model_name, tc.model_flavor)
        groups = {"dp_group": self.compute_group if self.world_size > 1 else None}
        cp = max(1, int(getattr(tc, "cp_degree", 1)))
        if cp > 1 and self.world_size > 1:
            # critic grouping: DP x CP (no TP / EP for the value net); rows are dealt over the DP index only
            from ..parallel.mesh import build_parallel_dims

            pd = build_parallel_dims(self.world_size, self.rank, dp_replicate=-1, dp_shard=1, cp=cp)
            self.parallel_dims = pd
            groups = {"dp_group": pd.batch_group, "cp_group": pd.cp_group, "loss_group": pd.loss_group}
        self.trainer = CriticTrainer(
            args, device=self.device, lr=c.lr, warmup_steps=c.warmup_steps, max_norm=c.max_norm,
            value_clip=c.value_clip, gamma=c.gamma, optimizer_kwargs=c.optimizer_kwargs, seq_len=tc.seq_len,
            max_tokens_per_micro=c.max_tokens_per_micro, train_backbone=c.train_backbone, **groups)
        if c.model_path and os.path.isdir(c.model_path):
            from ..models.hf import load_hf_checkpoint

            n = self.trainer.load_backbone(load_hf_checkpoint(args, c.model_path))
            log.info("critic backbone: %d tensors from %s", n, c.model_path)

    # ------------------------------------------------------------------ public (rank 0)
    def score_and_train(self, samples: list, publish: bool, global_step: int) -> dict | None:
        return self.submit_command("score_and_train", {"samples": samples, "publish": publish, "step": global_step})

    def offload(self) -> None:
        self.submit_command("offload", None)

    def restore(self) -> None:
        self.submit_command("restore", None)

    def on_colocate_acquire(self, grant) -> None:
        self.restore()

    def on_colocate_release(self, target: str) -> None:
        self.offload()

    # ------------------------------------------------------------------ collective
    def _my_rows(self, samples) -> list[int]:
        n = len(samples)
        lens = [len(s.tokens) for s in samples]
        order = sorted(range(n), key=lambda i: (-lens[i], i))
        pd = getattr(self, "parallel_dims", None)
        if pd is not None:  # CP ranks of one DP index share its rows
            return list(snake_deal(order, pd.dp)[pd.dp_rank])
        return list(snake_deal(order, self.world_size)[self.rank]) if self.world_size > 1 else list(range(n))

    def _gather(self, obj):
        if self.world_size == 1:
            return [obj]
        out = [None] * self.world_size if self.rank == 0 else None
        dist.gather_object(obj, out, dst=0, group=self.control_group)
        return out

    def cmd_score_and_train(self, payload) -> dict | None:
        samples = samples_from_rows(payload["samples"])
        rows = self._my_rows(samples)
        loss, values, metrics = self.trainer.train_window(samples, rows)
        for _ in range(max(0, int(self.cfg.value_epochs) - 1)):
            loss, _, metrics = self.trainer.train_window(samples, rows)
        self.windows += 1
        parts = self._gather({i: v for i, v in values.items()})
        step = int(payload["step"])
        if self.checkpoint.due(step) and self.runtime is not None:
            self.save_global_checkpoint(step)
        if self.rank != 0:
            return None
        allv: dict[int, torch.Tensor] = {}
        for p in parts:
            allv.update(p)
        vals = [allv[i] for i in range(len(samples))]
        first = []
        for s in samples:
            k = next((t for t, m in enumerate(s.mask) if m), 1) - 1
            first.append(max(0, k))
        v0 = [float(v[k]) if v.numel() > k else 0.0 for v, k in zip(vals, first)]
        v1 = [float(v[k + 1]) if v.numel() > k + 1 else v0[j] for j, (v, k) in enumerate(zip(vals, first))]
        rewards = [s.reward for s in samples]
        self.gauges.update(v0, rewards)
        diag = critic_diagnostics(v0, v1, rewards, split_by_prompt(samples))
        out: dict[str, Any] = {"value_loss": loss, "rows": len(samples), "diagnostics": diag,
                               "metrics": {**metrics, **diag.as_dict(), **self.gauges.as_dict()}}
        if payload["publish"]:
            if self.cfg.publish_mode == "values":
                out["values"] = [v.tolist() for v in vals]
            else:
                out["advantage"] = self._per_sequence_advantage(samples, vals)
        return out

    def _per_sequence_advantage(self, samples, vals) -> list[float]:
        from ..backend.gae import advantages_to_per_sequence, compute_vapo_gae
        from ..backend.critic.data import row_targets

        adv_out = []
        for s, v in zip(samples, vals):
            L = v.numel()
            mask, _ = row_targets(s, L, self.cfg.gamma)
            rew = torch.zeros(1, L)
            resp = (mask > 0).nonzero().flatten()
            if resp.numel():
                rew[0, int(resp[-1])] = s.reward
            a, _ = compute_vapo_gae(rew, v.view(1, L), mask.view(1, L), torch.zeros(1, L, dtype=torch.long), 1,
                                    gamma=self.cfg.gamma, alpha=self.cfg.alpha)
            adv_out.append(float(advantages_to_per_sequence(a, mask.view(1, L), torch.zeros(1, L, dtype=torch.long),
                                                            1)[0]))
        return adv_out

    def cmd_offload(self, payload) -> None:
        from ..backend.offload import offload_flat

        offload_flat(self.trainer.flat)

    def cmd_restore(self, payload) -> None:
        from ..backend.offload import restore_flat

        restore_flat(self.trainer.flat)

    # ------------------------------------------------------------------ checkpoints
    def save_global_checkpoint(self, step: int) -> None:
        store = self.runtime.state_store()
        d = store.shard_dir(self.service_name, step)
        os.makedirs(d, exist_ok=True)
        self.trainer.save_state(d)  # collective: every rank writes its share
        if self.rank == 0:
            store.write_meta(self.service_name, step, {"windows": self.windows, "train_steps": self.trainer.train_steps})
            store.mark_complete(self.service_name, step)
            store.prune(self.service_name, self.checkpoint.keep_latest_k)
        self.barrier()

    def restore_state(self, resume_step: int) -> bool:
        if resume_step <= 0 or self.runtime is None:
            return False
        store = self.runtime.state_store()
        if not store.is_complete(self.service_name, resume_step):
            raise FileNotFoundError(f"no critic shard at global step {resume_step}")
        self.trainer.load_state(store.shard_dir(self.service_name, resume_step))
        self.trainer.train_steps = int(store.payload(self.service_name, resume_step).get("train_steps", 0))
        self.windows = int(store.payload(self.service_name, resume_step)["windows"])
        return True


__all__ = ["CriticSpmdEngine"]
