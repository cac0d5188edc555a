"""Flat parameter, gradient and optimiser-state buffers.

All trainable tensors of a model live as views into a handful of contiguous
buffers (offsets padded to 128 bytes so every view is TMA-aligned):

* ``master``  fp32 — optimiser master weights;
* ``compute`` bf16 — what the kernels read (CUDA only; on CPU the module runs
  directly on ``master``);
* ``grad``    fp32 — ``param.main_grad`` views; wgrad GEMM epilogues
  accumulate into them;
* ``exp_avg`` / ``exp_avg_sq`` fp32 — AdamW moments.

One buffer per role makes the DDP gradient all-reduce one (bucketed)
collective over ``grad``, the optimiser one fused kernel over five flat
arrays (grad-norm scale, AdamW update, bf16 recast), and a weight sync one
copy of ``compute`` (or the recast written straight into an engine's
buffer).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn as nn

from ..ops._ext import ext
from ..ops.functional import native

ALIGN = 64  # elements; 128 B for bf16, 256 B for fp32


@dataclass
class Slot:
    name: str
    offset: int
    numel: int
    shape: tuple


def _align(n: int) -> int:
    return -(-n // ALIGN) * ALIGN


def flatten_module(module: nn.Module, dtype: torch.dtype, device) -> tuple[torch.Tensor, list[Slot]]:
    """Re-home every parameter of ``module`` into one flat ``dtype`` buffer.

    Same slot layout rule as :class:`FlatParams` (named-parameter order, offsets
    padded to ``ALIGN``), so a trainer's ``compute`` buffer and an engine's
    weight buffer can be copied into each other wholesale.
    """
    slots, off = [], 0
    params = list(module.named_parameters())
    for name, p in params:
        slots.append(Slot(name, off, p.numel(), tuple(p.shape)))
        off += _align(p.numel())
    flat = torch.zeros(off, dtype=dtype, device=device)
    with torch.no_grad():
        for s, (_, p) in zip(slots, params):
            view = flat[s.offset:s.offset + s.numel].view(s.shape)
            view.copy_(p.detach())
            p.data = view
    return flat, slots


class FlatParams:
    def __init__(self, model: nn.Module, *, compute_dtype: torch.dtype, device: torch.device,
                 keep_states: bool = True):
        self.device = torch.device(device)
        self.compute_dtype = compute_dtype
        self.slots: list[Slot] = []
        self.params: list[nn.Parameter] = []
        off = 0
        for name, p in model.named_parameters():
            self.slots.append(Slot(name, off, p.numel(), tuple(p.shape)))
            self.params.append(p)
            off += _align(p.numel())
        self.numel = off
        self.n_real = sum(s.numel for s in self.slots)
        dev = self.device
        self.master = torch.zeros(self.numel, dtype=torch.float32, device=dev)
        self.grad = torch.zeros(self.numel, dtype=torch.float32, device=dev)
        self.exp_avg = torch.zeros(self.numel, dtype=torch.float32, device=dev) if keep_states else None
        self.exp_avg_sq = torch.zeros(self.numel, dtype=torch.float32, device=dev) if keep_states else None
        self.separate_compute = compute_dtype != torch.float32
        self.compute = (torch.zeros(self.numel, dtype=compute_dtype, device=dev)
                        if self.separate_compute else self.master)
        with torch.no_grad():
            for s, p in zip(self.slots, self.params):
                self.master[s.offset:s.offset + s.numel].copy_(p.detach().reshape(-1).float())
                view = self.compute[s.offset:s.offset + s.numel].view(s.shape)
                if self.separate_compute:
                    view.copy_(p.detach().reshape(s.shape))
                p.data = view
                g = self.grad[s.offset:s.offset + s.numel].view(s.shape)
                if self.separate_compute:
                    p.main_grad = g
                    p.requires_grad_(True)
                else:
                    p.grad = g

    # ------------------------------------------------------------------
    def zero_grad(self) -> None:
        self.grad.zero_()
        if not self.separate_compute:
            for s, p in zip(self.slots, self.params):
                if p.grad is None or p.grad.data_ptr() != self.grad[s.offset:].data_ptr():
                    p.grad = self.grad[s.offset:s.offset + s.numel].view(s.shape)

    def collect_cpu_grads(self) -> None:
        """Fold gradients that autograd left in ``.grad`` into the flat fp32 buffer.

        The native GEMMs accumulate straight into ``main_grad`` and leave ``.grad`` empty. The PyTorch
        paths (the CPU oracle, and the library comparison baseline on CUDA) produce ordinary ``.grad``
        tensors: with a separate compute dtype they are added to ``main_grad`` in fp32 and dropped, so
        call this after every backward; without one ``.grad`` is re-pointed at the flat buffer."""
        if self.separate_compute:
            with torch.no_grad():
                for s, p in zip(self.slots, self.params):
                    if p.grad is not None:
                        p.main_grad.add_(p.grad)
                        p.grad = None
            return
        for s, p in zip(self.slots, self.params):
            view = self.grad[s.offset:s.offset + s.numel].view(s.shape)
            if p.grad is not None and p.grad.data_ptr() != view.data_ptr():
                view.copy_(p.grad)
                p.grad = view

    def view(self, buf: torch.Tensor, name: str) -> torch.Tensor:
        for s in self.slots:
            if s.name == name:
                return buf[s.offset:s.offset + s.numel].view(s.shape)
        raise KeyError(name)

    def gather_master(self) -> None:
        """Make every element of the fp32 master current on this rank when an optimiser shards it (a
        collective over the shard group: every rank of it must call this); a no-op otherwise."""
        shard = getattr(self, "master_shard", None)
        if shard is None:
            return
        import torch.distributed as dist

        lo, hi, group, per = shard
        world = dist.get_world_size(group)
        mine = torch.zeros(per, dtype=torch.float32, device=self.master.device)
        mine[:hi - lo].copy_(self.master[lo:hi])
        parts = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(parts, mine, group=group)
        with torch.no_grad():
            self.master.copy_(torch.cat(parts)[:self.numel])

    def state_dict(self, source: str = "master") -> dict[str, torch.Tensor]:
        """Weights by parameter name. ``source="master"``: the fp32 master (gathered first when sharded, a
        collective); ``"compute"``: the compute-dtype copy, which is complete on every rank."""
        if source == "compute":
            buf = self.compute
        else:
            self.gather_master()
            buf = self.master
        return {s.name: buf[s.offset:s.offset + s.numel].view(s.shape) for s in self.slots}

    @property
    def sync_source(self) -> torch.Tensor:
        """The buffer a weight sync reads: the compute-dtype copy (complete on every rank, and what the
        inference engines hold) when there is one, else the fp32 master."""
        return self.compute if self.separate_compute else self.master

    def load_state_dict(self, sd: dict[str, torch.Tensor]) -> None:
        with torch.no_grad():
            for s in self.slots:
                self.master[s.offset:s.offset + s.numel].copy_(sd[s.name].reshape(-1).float())
            self.recast()

    def recast(self) -> None:
        if self.separate_compute:
            self.compute.copy_(self.master)

    # ------------------------------------------------------------------
    def grad_norm(self) -> torch.Tensor:
        """Global L2 norm of ``grad`` (device scalar, no host sync)."""
        if self.grad.is_cuda and native(self.grad):
            out = torch.zeros(1, dtype=torch.float32, device=self.device)
            ext().sq_norm(self.grad, out)
            return out.sqrt().reshape(())
        return self.grad.double().norm().float()  # fp64 accumulation: the CPU oracle's norm is exact to fp32


class FlatAdamW:
    """AdamW over :class:`FlatParams` with global-norm clipping.

    The clip coefficient stays on the device: the CUDA path reads it inside the
    update kernel, so a step has no host synchronisation.  ``mirror`` names an
    extra compute-dtype buffer (e.g. a colocated rollout engine's weights in
    the same layout) that the update writes alongside ``compute``.
    """

    def __init__(self, flat: FlatParams, *, lr: float, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 0.0, max_norm: float = 1.0):
        self.flat = flat
        self.lr = lr
        self.base_lr = lr
        self.betas = betas
        self.eps = eps
        self.weight_decay = weight_decay
        self.max_norm = max_norm
        self.step_count = 0
        self.mirror: torch.Tensor | None = None

    def set_decay_slots(self, names) -> None:
        """Apply weight decay only to the named parameters (a decay / no-decay grouping); ``None`` restores
        decay on every parameter."""
        if names is None:
            self.decay_names = None
            return
        wanted = set(names)
        self.decay_names = [s.name for s in self.flat.slots if s.name in wanted]

    def _decay_views(self):
        f = self.flat
        if hasattr(f, "shard_views"):  # sharded parameters: this rank's pieces of them
            return f.shard_views(f.master, self.decay_names)
        by_name = {s.name: s for s in f.slots}
        return [f.master[by_name[n].offset:by_name[n].offset + by_name[n].numel] for n in self.decay_names]

    def step(self, grad_norm: torch.Tensor | None = None) -> torch.Tensor:
        try:
            return self._grouped_step(grad_norm)
        finally:
            changed = getattr(self.flat, "weights_changed", None)
            if changed is not None:  # sharded parameters: gathered copies are stale now
                changed()

    def _grouped_step(self, grad_norm: torch.Tensor | None) -> torch.Tensor:
        f = self.flat
        if grad_norm is None:
            grad_norm = f.grad_norm()
        if getattr(self, "decay_names", None) is not None:
            # grouped decay: the decoupled factor (1 - lr * wd) multiplies the decaying parameters before an
            # update without decay -- the same result as AdamW with per-group weight decay
            wd = self.weight_decay
            self.weight_decay = 0.0
            try:
                with torch.no_grad():
                    views = self._decay_views()
                    if views and wd:
                        torch._foreach_mul_(views, 1.0 - self.lr * wd)
                return self._step(grad_norm)
            finally:
                self.weight_decay = wd
        return self._step(grad_norm)

    def _step(self, grad_norm: torch.Tensor) -> torch.Tensor:
        f = self.flat
        self.step_count += 1
        b1, b2 = self.betas
        if f.grad.is_cuda and not native(f.grad):
            self._library_step(grad_norm)
        elif f.grad.is_cuda:
            ext().adamw_flat(f.master, f.grad, f.exp_avg, f.exp_avg_sq,
                             f.compute if f.separate_compute else None, self.mirror, grad_norm.reshape(1),
                             float(self.max_norm), float(self.lr), float(b1), float(b2), float(self.eps),
                             float(self.weight_decay), int(self.step_count))
        else:
            from ..ops.reference import adamw_

            scale = 1.0
            if self.max_norm and self.max_norm > 0:
                gn = float(grad_norm)
                scale = min(1.0, self.max_norm / (gn + 1e-6)) if math.isfinite(gn) else 1.0
            with torch.no_grad():
                adamw_(f.master, f.grad, f.exp_avg, f.exp_avg_sq, lr=self.lr, beta1=b1, beta2=b2, eps=self.eps,
                       weight_decay=self.weight_decay, step=self.step_count, grad_scale=scale)
                if f.separate_compute:
                    f.compute.copy_(f.master)
                if self.mirror is not None:
                    self.mirror.copy_(f.master)
        return grad_norm

    def _library_step(self, grad_norm: torch.Tensor) -> None:
        """Comparison baseline only: ``clip_grad_norm_``-style scaling and PyTorch's fused AdamW kernel over
        the flat fp32 buffers, then a cast copy into the compute weights."""
        f = self.flat
        b1, b2 = self.betas
        with torch.no_grad():
            if self.max_norm and self.max_norm > 0:
                coef = (self.max_norm / (grad_norm.float() + 1e-6)).clamp(max=1.0)
                f.grad.mul_(coef)
            if not hasattr(self, "_step_t"):
                self._step_t = torch.zeros((), dtype=torch.float32, device=f.grad.device)
            self._step_t.fill_(float(self.step_count))  # the fused kernel reads the already-advanced step
            torch._fused_adamw_([f.master], [f.grad], [f.exp_avg], [f.exp_avg_sq], [], [self._step_t],
                                lr=self.lr, beta1=b1, beta2=b2, weight_decay=self.weight_decay, eps=self.eps,
                                amsgrad=False, maximize=False)
            if f.separate_compute:
                f.compute.copy_(f.master)
            if self.mirror is not None:
                self.mirror.copy_(f.master)

    def state_dict(self) -> dict:
        return {"step": self.step_count, "exp_avg": self.flat.exp_avg, "exp_avg_sq": self.flat.exp_avg_sq,
                "lr": self.lr}

    def load_state_dict(self, sd: dict) -> None:
        self.step_count = int(sd["step"])
        self.flat.exp_avg.copy_(sd["exp_avg"])
        self.flat.exp_avg_sq.copy_(sd["exp_avg_sq"])
        self.lr = float(sd.get("lr", self.lr))


def lr_lambda(step: int, *, warmup: int, total: int, decay_ratio: float | None, decay_type: str,
              min_factor: float) -> float:
    """Warmup → stable → decay multiplier (reference ``TrainerConfig`` lr knobs)."""
    if warmup > 0 and step < warmup:
        return (step + 1) / (warmup + 1)
    if decay_ratio == 0.0:
        return 1.0
    if decay_ratio is None:
        decay_start, decay_steps = warmup, max(1, total - warmup)
    else:
        decay_steps = max(1, int(round(total * decay_ratio)))
        decay_start = total - decay_steps
    if step < decay_start:
        return 1.0
    prog = min(1.0, (step - decay_start) / decay_steps)
    if decay_type == "linear":
        f = 1.0 - prog
    elif decay_type == "sqrt":
        f = 1.0 - math.sqrt(prog)
    else:
        f = 0.5 * (1.0 + math.cos(math.pi * prog))
    return min_factor + (1.0 - min_factor) * f


__all__ = ["FlatAdamW", "FlatParams", "lr_lambda"]
