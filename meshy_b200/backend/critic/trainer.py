"""Critic value training: one optimiser step per window, accumulated over micro-batches.

Behaviour of the reference's ``CriticEngine.train_value_accumulated``
(``meshy/backend/titan/critic/engine.py:493-655``):

* the loss is the masked clipped squared value error summed over every
  micro-batch of the window divided by the *global* count of response tokens
  (all micro-batches, all DP ranks), so the summed DP gradient equals the
  gradient of the window mean while peak memory stays at one micro-batch;
* every forward of the window runs on the pre-update weights, so the values
  it returns are the ones a separate scoring pass would give -- they are what
  gets published (values mode) or turned into advantages;
* linear learning-rate warmup over ``warmup_steps`` windows, global-norm
  clipping, a non-finite loss raises.

B200 layout: the backbone lives in flat buffers (bf16 compute, fp32 master,
gradients accumulated by the wgrad GEMM epilogues, one AdamW kernel); the
fp32 value head has its own tiny optimiser; the DP gradient reduction is the
same flat-buffer reducer the actor uses.
"""

from __future__ import annotations

import math
from typing import Sequence

import torch
import torch.distributed as dist

from ...models.args import ModelArgs
from ...parallel.ddp import GradReducer
from ..flat import FlatAdamW, FlatParams
from ..vapo import clipped_value_error
from .data import CriticMicro, TrajectorySample, pack_micros
from .model import CriticModel


class CriticTrainer:
    def __init__(self, args: ModelArgs, *, device="cpu", lr: float = 5e-6, warmup_steps: int = 10,
                 max_norm: float = 1.0, value_clip: float | None = None, gamma: float = 1.0,
                 weight_decay: float = 0.0, betas=(0.9, 0.999), eps: float = 1e-8, seq_len: int = 8192,
                 max_tokens_per_micro: int | None = None, dp_group=None, train_backbone: bool = True, seed: int = 0,
                 model: CriticModel | None = None):
        self.args = args
        self.device = torch.device(device)
        self.dp_group = dp_group
        self.seq_len = seq_len
        self.max_tokens = max_tokens_per_micro
        self.gamma = gamma
        self.value_clip = value_clip
        self.warmup_steps = int(warmup_steps)
        self.max_norm = max_norm
        self.base_lr = lr
        self.train_backbone = train_backbone
        self.model = model if model is not None else CriticModel(args, seed=seed, device=self.device)
        cdt = torch.bfloat16 if self.device.type == "cuda" else torch.float32
        self.flat = FlatParams(self.model.backbone, compute_dtype=cdt, device=self.device)
        self.opt = FlatAdamW(self.flat, lr=lr, betas=betas, eps=eps, weight_decay=weight_decay, max_norm=0.0)
        self.head_opt = torch.optim.AdamW([self.model.value_head, self.model.value_bias], lr=lr, betas=betas,
                                          eps=eps, weight_decay=0.0)
        self.reducer = GradReducer(self.flat, dp_group)
        self.train_steps = 0

    # ------------------------------------------------------------------ helpers
    @property
    def dp_world(self) -> int:
        if self.dp_group is None or not dist.is_initialized():
            return 1
        return dist.get_world_size(self.dp_group)

    def _all_sum(self, x: torch.Tensor) -> torch.Tensor:
        if self.dp_world > 1:
            dev = self.device if dist.get_backend(self.dp_group) == "nccl" else torch.device("cpu")
            y = x.detach().to(dev).clone()
            dist.all_reduce(y, group=self.dp_group)
            return y.to(x.device)
        return x

    def _micros(self, samples: Sequence[TrajectorySample], rows: Sequence[int]) -> list[CriticMicro]:
        return pack_micros(samples, rows, self.seq_len, self.max_tokens, self.gamma)

    def _forward(self, mb: CriticMicro) -> torch.Tensor:
        d = self.device
        return self.model(mb.input_ids.to(d), mb.positions.to(d), mb.cu_seqlens.to(d), mb.max_seqlen)

    def _split_values(self, mb: CriticMicro, v: torch.Tensor) -> dict[int, torch.Tensor]:
        out, off = {}, 0
        for r, L in zip(mb.rows, mb.lengths):
            out[r] = v[off:off + L].detach().float().cpu()
            off += L
        return out

    # ------------------------------------------------------------------ public
    @torch.no_grad()
    def predict(self, samples: Sequence[TrajectorySample], rows: Sequence[int]) -> dict[int, torch.Tensor]:
        out: dict[int, torch.Tensor] = {}
        for mb in self._micros(samples, rows):
            out.update(self._split_values(mb, self._forward(mb)))
        return out

    def _apply_warmup(self) -> float:
        scale = 1.0 if self.warmup_steps <= 0 else min(1.0, self.train_steps / self.warmup_steps)
        lr = self.base_lr * scale
        self.opt.lr = lr
        for g in self.head_opt.param_groups:
            g["lr"] = lr
        return lr

    def train_window(self, samples: Sequence[TrajectorySample], rows: Sequence[int],
                     old_values: dict[int, torch.Tensor] | None = None) -> tuple[float, dict[int, torch.Tensor], dict]:
        """One value step over ``rows`` (this rank's share of the window); returns the window loss,
        the pre-update values of ``rows`` and step metrics."""
        self.train_steps += 1
        lr = self._apply_warmup()
        micros = self._micros(samples, rows)
        local_cnt = torch.tensor(float(sum(float(mb.mask.sum()) for mb in micros)))
        denom = float(self._all_sum(local_cnt).clamp(min=1.0))
        self.flat.zero_grad()
        self.head_opt.zero_grad(set_to_none=False)
        for p in (self.model.value_head, self.model.value_bias):
            if p.grad is None:
                p.grad = torch.zeros_like(p)
        values: dict[int, torch.Tensor] = {}
        num = torch.zeros((), dtype=torch.float64)
        d = self.device
        for mb in micros:
            with torch.set_grad_enabled(True):
                if self.train_backbone:
                    v = self._forward(mb)
                else:
                    with torch.no_grad():
                        h = self.model.backbone.hidden(mb.input_ids.to(d), mb.positions.to(d),
                                                       mb.cu_seqlens.to(d), mb.max_seqlen)
                    v = (h.float() @ self.model.value_head.t()).squeeze(-1) + self.model.value_bias
                old = None
                if old_values is not None:
                    old = torch.cat([old_values[r][:L] for r, L in zip(mb.rows, mb.lengths)]).to(d)
                elif self.value_clip is not None:
                    old = v.detach()
                err = clipped_value_error(v, mb.returns.to(d), old, self.value_clip) * mb.mask.to(d)
                numer = err.sum()
                loss = numer / denom
                if not torch.isfinite(loss):
                    raise RuntimeError(f"non-finite critic loss: {float(loss)}")
                loss.backward()
            num += float(numer.detach())
            values.update(self._split_values(mb, v))
        self.flat.collect_cpu_grads()
        if self.train_backbone:
            self.reducer.finish()
        head = torch.cat([self.model.value_head.grad.reshape(-1), self.model.value_bias.grad.reshape(-1)])
        head = self._all_sum(head)
        self.model.value_head.grad.copy_(head[:-1].view_as(self.model.value_head))
        self.model.value_bias.grad.copy_(head[-1:])
        gn_bb = self.flat.grad_norm().float().cpu() if self.train_backbone else torch.zeros(())
        gn = math.sqrt(float(gn_bb) ** 2 + float(head.float().norm()) ** 2)
        scale = 1.0
        if self.max_norm and self.max_norm > 0 and math.isfinite(gn):
            scale = min(1.0, self.max_norm / (gn + 1e-6))
        if self.train_backbone:
            if scale < 1.0:
                self.flat.grad.mul_(scale)
            self.opt.step(grad_norm=torch.zeros((), device=self.flat.grad.device))
        with torch.no_grad():
            self.model.value_head.grad.mul_(scale)
            self.model.value_bias.grad.mul_(scale)
        self.head_opt.step()
        window_loss = float(self._all_sum(torch.tensor(float(num))) / denom)
        return window_loss, values, {"critic/value_loss": window_loss, "critic/grad_norm": gn, "critic/lr": lr,
                                     "critic/tokens": denom}

    # ------------------------------------------------------------------ state
    def state_dict(self) -> dict:
        return {"flat": self.flat.state_dict(), "opt": self.opt.state_dict(),
                "head": {"w": self.model.value_head.detach().cpu(), "b": self.model.value_bias.detach().cpu()},
                "head_opt": self.head_opt.state_dict(), "train_steps": self.train_steps}

    def load_state_dict(self, sd: dict) -> None:
        self.flat.load_state_dict(sd["flat"])
        self.opt.load_state_dict(sd["opt"])
        with torch.no_grad():
            self.model.value_head.copy_(sd["head"]["w"])
            self.model.value_bias.copy_(sd["head"]["b"])
        self.head_opt.load_state_dict(sd["head_opt"])
        self.train_steps = int(sd["train_steps"])

    def load_backbone(self, state: dict[str, torch.Tensor]) -> int:
        """Backbone weights from an actor/HF state dict (the LM head and value head are skipped)."""
        mine = {s.name for s in self.flat.slots}
        sd = {k: v for k, v in state.items() if k in mine}
        missing = mine - set(sd)
        if missing:
            raise KeyError(f"backbone weights missing: {sorted(missing)[:5]}")
        self.flat.load_state_dict(sd)
        return len(sd)


__all__ = ["CriticTrainer"]
