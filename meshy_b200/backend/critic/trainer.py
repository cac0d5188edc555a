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

Optimiser grouping follows the reference critic (``critic/engine.py:158-168``,
``vapo.py:44-50``): without ``optimizer_kwargs`` one AdamW group with PyTorch's
defaults (weight decay 0.01 on every parameter); with them, a decay group
(matrices, ``weight_decay`` from the kwargs, default 0.01) and a no-decay group
(vectors and biases), and those explicit settings stay authoritative when a
checkpoint with another grouping is restored (:meth:`load_state`).
"""

from __future__ import annotations

import math
from typing import Sequence

import torch
import torch.distributed as dist

from ...models.args import ModelArgs
from ...parallel.ddp import GradReducer
from ..flat import FlatAdamW, FlatParams
from .data import CriticMicro, TrajectorySample, pack_micros
from .model import CriticModel, value_head_loss


class CriticTrainer:
    def __init__(self, args: ModelArgs, *, device="cpu", lr: float = 5e-6, warmup_steps: int = 10,
                 max_norm: float = 1.0, value_clip: float | None = None, gamma: float = 1.0,
                 optimizer_kwargs: dict | None = None, seq_len: int = 8192,
                 max_tokens_per_micro: int | None = None, dp_group=None, train_backbone: bool = True, seed: int = 0,
                 model: CriticModel | None = None, cp_group=None, loss_group=None):
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
        opts = dict(optimizer_kwargs or {})
        wd = float(opts.pop("weight_decay", 0.01))
        betas = tuple(opts.pop("betas", (0.9, 0.999)))
        eps = float(opts.pop("eps", 1e-8))
        #: explicit optimiser settings win over a restored checkpoint's (grouping and hyperparameters)
        self.restore_optimizer_config = optimizer_kwargs is not None
        self.grouped = optimizer_kwargs is not None
        self.opt = FlatAdamW(self.flat, lr=lr, betas=betas, eps=eps, weight_decay=wd, max_norm=0.0)
        if self.grouped:
            self.opt.set_decay_slots(s.name for s in self.flat.slots if len(s.shape) >= 2)
            head_groups = [{"params": [self.model.value_head], "weight_decay": wd},
                           {"params": [self.model.value_bias], "weight_decay": 0.0}]
        else:
            head_groups = [{"params": [self.model.value_head, self.model.value_bias], "weight_decay": wd}]
        self.head_opt = torch.optim.AdamW(head_groups, lr=lr, betas=betas, eps=eps)
        # context parallelism: every row of a micro-batch is padded to a multiple of 2 x cp and split head-tail
        # over the CP group (reference ``critic/engine.py:561-618``); gradients then sum over DP x CP
        self.cp = None
        if cp_group is not None and dist.is_initialized() and dist.get_world_size(cp_group) > 1:
            from ...parallel.cp import CpSharder

            self.cp = CpSharder(cp_group)
        self.loss_group = loss_group if loss_group is not None else dp_group
        self.reducer = GradReducer(self.flat, self.loss_group)
        if self.reducer.overlapping and self.train_backbone:
            self.model.backbone.block_hooks = self.reducer  # per-block all-reduce in the last micro's backward
        self.train_steps = 0

    # ------------------------------------------------------------------ helpers
    @property
    def dp_world(self) -> int:
        if self.dp_group is None or not dist.is_initialized():
            return 1
        return dist.get_world_size(self.dp_group)

    def _all_sum(self, x: torch.Tensor, group=None) -> torch.Tensor:
        g = self.dp_group if group is None else group
        if g is not None and dist.is_initialized() and dist.get_world_size(g) > 1:
            dev = self.device if dist.get_backend(g) == "nccl" else torch.device("cpu")
            y = x.detach().to(dev).clone()
            dist.all_reduce(y, group=g)
            return y.to(x.device)
        return x

    def _micros(self, samples: Sequence[TrajectorySample], rows: Sequence[int]) -> list[CriticMicro]:
        return pack_micros(samples, rows, self.seq_len, self.max_tokens, self.gamma)

    def _forward(self, mb: CriticMicro) -> torch.Tensor:
        d = self.device
        if getattr(mb, "cp_layout", None) is not None:
            from ...parallel.cp import cp_attention

            with cp_attention(self.cp, mb.cp_layout):
                return self.model(mb.input_ids.to(d), mb.positions.to(d), mb.cu_seqlens.to(d), mb.max_seqlen)
        return self.model(mb.input_ids.to(d), mb.positions.to(d), mb.cu_seqlens.to(d), mb.max_seqlen)

    def _hidden(self, mb: CriticMicro) -> torch.Tensor:
        """Final normed hidden states of a micro-batch (the value head's input)."""
        d = self.device
        args = (mb.input_ids.to(d), mb.positions.to(d), mb.cu_seqlens.to(d), mb.max_seqlen)
        if getattr(mb, "cp_layout", None) is not None:
            from ...parallel.cp import cp_attention

            with cp_attention(self.cp, mb.cp_layout):
                return self.model.backbone.hidden(*args)
        return self.model.backbone.hidden(*args)

    def _cp_shard(self, mb: CriticMicro) -> CriticMicro:
        """Pad every row of a packed micro-batch to one length divisible by 2 x cp and keep this CP rank's
        head-tail chunks (ids, positions, mask and returns alike)."""
        from ...parallel.cp import CpLayout

        rows = len(mb.rows)
        div = 2 * self.cp.size
        S = -(-mb.max_seqlen // div) * div
        def pad(t, fill=0):
            out = torch.full((rows, S), fill, dtype=t.dtype)
            off = 0
            for r, L in enumerate(mb.lengths):
                out[r, :L] = t[off:off + L]
                off += L
            return out
        ids, msk, ret = pad(mb.input_ids), pad(mb.mask), pad(mb.returns)
        pos = torch.arange(S, dtype=torch.int32).repeat(rows, 1)
        ids, pos, msk, ret = self.cp.shard_seq(ids, pos, msk, ret)
        L = ids.shape[1]
        sh = CriticMicro(mb.rows, ids.reshape(-1), pos.reshape(-1),
                         torch.arange(0, rows * L + 1, L, dtype=torch.int32), L, msk.reshape(-1), ret.reshape(-1),
                         list(mb.lengths))
        sh.cp_layout = CpLayout(rows, S, S // div)
        return sh

    def _values_of(self, mb: CriticMicro, v: torch.Tensor) -> dict[int, torch.Tensor]:
        """Per-row values of a micro-batch (a CP micro gathers the full rows from the CP group first)."""
        if getattr(mb, "cp_layout", None) is None:
            return self._split_values(mb, v)
        rows = len(mb.rows)
        (full,) = self.cp.gather_seq(v.detach().view(rows, -1))
        return {r: full[j, :L].float().cpu() for j, (r, L) in enumerate(zip(mb.rows, mb.lengths))}

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
            if self.cp is not None:
                mb = self._cp_shard(mb)
            out.update(self._values_of(mb, self._forward(mb)))
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
        # the denominator counts every response token of the window once (full rows, summed over DP)
        # with it, how many DP ranks have a micro-batch: the per-block gradient all-reduces started inside the
        # last micro's backward only line up across ranks when every rank runs one
        local = torch.tensor([float(sum(float(mb.mask.sum()) for mb in micros)), 1.0 if micros else 0.0])
        tot = self._all_sum(local)
        denom = float(tot[0].clamp(min=1.0))
        overlap = self.train_backbone and self.reducer.overlapping and int(tot[1]) == self.dp_world
        if self.cp is not None:
            micros = [self._cp_shard(mb) for mb in micros]
        self.flat.zero_grad()
        self.head_opt.zero_grad(set_to_none=False)
        for p in (self.model.value_head, self.model.value_bias):
            if p.grad is None:
                p.grad = torch.zeros_like(p)
        values: dict[int, torch.Tensor] = {}
        num = torch.zeros((), dtype=torch.float64)
        d = self.device
        for i, mb in enumerate(micros):
            if overlap and i == len(micros) - 1:
                self.reducer.arm()
            with torch.set_grad_enabled(True):
                with torch.set_grad_enabled(self.train_backbone):
                    h = self._hidden(mb)
                old = None
                if old_values is not None and self.cp is not None:
                    raise NotImplementedError("explicit old values with context parallelism")
                if old_values is not None:
                    old = torch.cat([old_values[r][:L] for r, L in zip(mb.rows, mb.lengths)]).to(d)
                elif self.value_clip is not None:
                    # this window's own forward is the old value of its clipping (pre-update weights)
                    with torch.no_grad():
                        _, old = value_head_loss(h.detach(), self.model.value_head, self.model.value_bias,
                                                 mb.returns.to(d), mb.mask.to(d), None, None, 1.0)
                loss, v = value_head_loss(h, self.model.value_head, self.model.value_bias, mb.returns.to(d),
                                          mb.mask.to(d), old, self.value_clip, denom)
                if not torch.isfinite(loss):
                    raise RuntimeError(f"non-finite critic loss: {float(loss)}")
                loss.backward()
            num += float(loss.detach()) * denom
            values.update(self._values_of(mb, v))
        self.flat.collect_cpu_grads()
        if self.train_backbone:
            self.reducer.finish()
        head = torch.cat([self.model.value_head.grad.reshape(-1), self.model.value_bias.grad.reshape(-1)])
        head = self._all_sum(head, self.loss_group)
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
        window_loss = float(self._all_sum(torch.tensor(float(num)), self.loss_group) / denom)
        return window_loss, values, {"critic/value_loss": window_loss, "critic/grad_norm": gn, "critic/lr": lr,
                                     "critic/tokens": denom}

    # ------------------------------------------------------------------ DCP state (reference layout)
    def _fqn_slots(self):
        """(torchtitan FQN, backbone slot, piece shape) of every backbone tensor, in slot order."""
        from ...models.titan_names import titan_pieces

        out = []
        for s in self.flat.slots:
            for fqn, t in titan_pieces(self.args, s.name, torch.empty(s.shape, device="meta")):
                out.append((fqn, s, tuple(t.shape)))
        return out

    def _pieces(self, buf: torch.Tensor, s):
        from ...models.titan_names import titan_pieces

        return [t for _, t in titan_pieces(self.args, s.name, buf[s.offset:s.offset + s.numel].view(s.shape))]

    def _groups_doc(self) -> list[dict]:
        """param_groups as PyTorch's FQN-keyed state dict writes them."""
        o = self.opt
        base = {"lr": float(o.lr), "betas": tuple(float(b) for b in o.betas), "eps": float(o.eps), "amsgrad": False,
                "maximize": False}
        fqns = [(q, s, None) for q, s, _ in self._fqn_slots()]
        if not self.grouped:
            return [dict(base, weight_decay=float(o.weight_decay),
                         params=[q for q, _, _ in fqns] + ["value_head.weight", "value_head.bias"])]
        decay = set(o.decay_names or [])
        return [dict(base, weight_decay=float(o.weight_decay),
                     params=[q for q, s, _ in fqns if s.name in decay] + ["value_head.weight"]),
                dict(base, weight_decay=0.0, params=[q for q, s, _ in fqns if s.name not in decay] +
                     ["value_head.bias"])]

    def save_state(self, path: str) -> None:
        """The critic's value net and AdamW state as DCP ``{"model": ..., "optim": {"state", "param_groups"}}``
        under torchtitan FQNs (``value_head.weight`` / ``value_head.bias`` for the head), as the reference
        critic writes it. Collective over the DP group: each rank writes the parameters it owns."""
        import torch.distributed.checkpoint as dcp

        from ..checkpoint import _owners

        self.flat.gather_master()
        if self.cp is not None and self.cp.rank != 0:
            return  # CP ranks hold the same weights; the first rank of each CP group writes
        world = self.dp_world
        rank = dist.get_rank(self.dp_group) if world > 1 else 0
        owner = _owners(self.flat.slots, world)
        f, n = self.flat, float(self.opt.step_count)
        model, state = {}, {}
        names_of: dict = {}
        for q, s, _ in self._fqn_slots():
            names_of.setdefault(s.name, []).append(q)
        for s, who in zip(f.slots, owner):
            if who != rank:
                continue
            for q, w, m, v in zip(names_of[s.name], self._pieces(f.master, s), self._pieces(f.exp_avg, s),
                                  self._pieces(f.exp_avg_sq, s)):
                model[q] = w.detach().float().cpu().contiguous()
                state[q] = {"step": torch.tensor(n), "exp_avg": m.detach().float().cpu().contiguous(),
                            "exp_avg_sq": v.detach().float().cpu().contiguous()}
        if rank == 0:
            head = {"value_head.weight": self.model.value_head, "value_head.bias": self.model.value_bias}
            for q, p in head.items():
                model[q] = p.detach().float().cpu().clone()
                st = self.head_opt.state.get(p, {})
                state[q] = {"step": torch.tensor(float(st["step"]) if "step" in st else 0.0),
                            "exp_avg": st.get("exp_avg", torch.zeros_like(p)).detach().float().cpu().clone(),
                            "exp_avg_sq": st.get("exp_avg_sq", torch.zeros_like(p)).detach().float().cpu().clone()}
        doc = {"model": model, "optim": {"state": state}}
        if rank == 0:
            doc["optim"]["param_groups"] = self._groups_doc()
        group = self.dp_group if world > 1 else None
        dcp.save(doc, checkpoint_id=path, process_group=group, no_dist=group is None)

    def load_state(self, path: str) -> None:
        """Restore what :meth:`save_state` wrote (or the reference critic's checkpoint). Moments and steps are
        matched by parameter name, whatever grouping the checkpoint had. With explicit ``optimizer_kwargs`` the
        current groups and hyperparameters stay; without them the saved hyperparameters are applied."""
        import os

        import torch.distributed.checkpoint as dcp

        from ...models.titan_names import join_pieces

        if not os.path.isdir(path):
            raise FileNotFoundError(f"not a critic checkpoint directory: {path}")
        f = self.flat
        plan: dict = {}
        want_model, want_state = {}, {}
        for q, s, shape in self._fqn_slots():
            plan.setdefault(s.name, (s, []))[1].append(q)
            want_model[q] = torch.empty(shape, dtype=torch.float32)
            want_state[q] = {"step": torch.tensor(0.0), "exp_avg": torch.empty(shape, dtype=torch.float32),
                             "exp_avg_sq": torch.empty(shape, dtype=torch.float32)}
        for q, p in (("value_head.weight", self.model.value_head), ("value_head.bias", self.model.value_bias)):
            want_model[q] = torch.empty(p.shape, dtype=torch.float32)
            want_state[q] = {"step": torch.tensor(0.0), "exp_avg": torch.empty(p.shape, dtype=torch.float32),
                             "exp_avg_sq": torch.empty(p.shape, dtype=torch.float32)}
        doc = {"model": want_model, "optim": {"state": want_state}}
        if not self.restore_optimizer_config:
            from torch.distributed.checkpoint import FileSystemReader

            meta = FileSystemReader(path).read_metadata().state_dict_metadata
            if any(k.startswith("optim.param_groups") for k in meta):
                doc["optim"]["param_groups"] = self._groups_doc()
        group = self.dp_group if self.dp_world > 1 else None
        dcp.load(doc, checkpoint_id=path, process_group=group, no_dist=group is None)
        steps = 0
        with torch.no_grad():
            for name, (s, qs) in plan.items():
                f.master[s.offset:s.offset + s.numel].copy_(join_pieces(self.args, name, [want_model[q] for q in qs])
                                                            .reshape(-1))
                f.exp_avg[s.offset:s.offset + s.numel].copy_(
                    join_pieces(self.args, name, [want_state[q]["exp_avg"] for q in qs]).reshape(-1))
                f.exp_avg_sq[s.offset:s.offset + s.numel].copy_(
                    join_pieces(self.args, name, [want_state[q]["exp_avg_sq"] for q in qs]).reshape(-1))
                steps = max(steps, int(float(want_state[qs[0]]["step"])))
            f.recast()
            for q, p in (("value_head.weight", self.model.value_head), ("value_head.bias", self.model.value_bias)):
                p.copy_(want_model[q].reshape(p.shape))
                st = want_state[q]
                self.head_opt.state[p] = {"step": st["step"].clone(), "exp_avg": st["exp_avg"].to(p.device).clone(),
                                          "exp_avg_sq": st["exp_avg_sq"].to(p.device).clone()}
        self.opt.step_count = steps
        groups = doc["optim"].get("param_groups")
        if groups and not self.restore_optimizer_config:
            g0 = groups[0]
            self.opt.betas = tuple(g0["betas"])
            self.opt.eps = float(g0["eps"])
            self.opt.weight_decay = float(g0["weight_decay"])
            for hg in self.head_opt.param_groups:
                hg["betas"], hg["eps"] = tuple(g0["betas"]), float(g0["eps"])

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
