"""Symmetric peer memory over NVLink and the fused data-parallel optimiser step.

:class:`SymmetricHeap` — every rank of a single-node process group allocates
the same number of bytes (``cudaMalloc``, zeroed), exports a CUDA IPC handle,
all-gathers the handles over the group, and maps every peer's buffer.  The
device-side pointer tables (one int64 per rank) are what kernels index with a
rank number; slot ``rank`` holds the local pointer.  Views into the heap are
plain torch tensors (non-owning; the heap object keeps the memory alive).

:class:`FusedDPAdamW` — the DDP gradient reduction and the optimiser step as
one device pipeline over peer memory (``csrc/kernels/symm.cu``):
reduce-scatter of the fp32 gradient straight from the peers' buffers, global
gradient norm, clip + AdamW on this rank's shard with local moments, and the
all-gather of the new fp32 master / bf16 compute weights by P2P stores into
every rank's buffers.  It replaces "NCCL all-reduce of the whole gradient +
a full-size AdamW on every rank" (the reference's DDP path: fp32 all-reduce,
``TT:torchtitan/config/configs.py:64``) and produces the same update.

Flat buffers are re-homed into the heap (master, grad, compute); their
current contents are kept.  Waits inside the kernels are bounded: a peer that
never arrives makes the step raise instead of hanging the GPU.
"""

from __future__ import annotations

import os

import torch
import torch.distributed as dist

from ..ops._ext import ext

_DTYPE_SIZE = {torch.float32: 4, torch.bfloat16: 2, torch.int32: 4, torch.int64: 8, torch.uint8: 1}


def _align(n: int, a: int = 256) -> int:
    return -(-n // a) * a


class SymmetricHeap:
    """One region per rank, mapped by every rank; regions are carved with :meth:`alloc`."""

    def __init__(self, nbytes: int, group=None, device: torch.device | None = None):
        if not (dist.is_initialized()):
            raise RuntimeError("SymmetricHeap needs an initialised process group")
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.nbytes = _align(int(nbytes))
        C = ext()
        with torch.cuda.device(self.device):
            self.base = C.symm_alloc(self.nbytes)
            handle = C.symm_export(self.base)
        handles: list = [None] * self.world
        dist.all_gather_object(handles, (self.rank, handle), group=group)
        self.ptrs = [0] * self.world
        self._opened = []
        with torch.cuda.device(self.device):
            for r, h in handles:
                if r == self.rank:
                    self.ptrs[r] = self.base
                else:
                    p = C.symm_import(h)
                    self.ptrs[r] = p
                    self._opened.append(p)
        self._used = 0

    def alloc(self, numel: int, dtype: torch.dtype) -> tuple[torch.Tensor, torch.Tensor]:
        """A symmetric region: (local tensor view, device int64 table of every rank's address)."""
        nb = _align(numel * _DTYPE_SIZE[dtype])
        if self._used + nb > self.nbytes:
            raise RuntimeError(f"symmetric heap exhausted ({self._used + nb} > {self.nbytes} bytes)")
        off = self._used
        self._used += nb
        with torch.cuda.device(self.device):
            view = ext().symm_view(self.base, off, numel, dtype)
        table = torch.tensor([p + off for p in self.ptrs], dtype=torch.int64, device=self.device)
        return view, table

    def close(self) -> None:
        C = ext()
        for p in self._opened:
            try:
                C.symm_close(p)
            except Exception:
                pass
        self._opened = []
        if self.base:
            torch.cuda.synchronize(self.device)
            C.symm_free(self.base)
            self.base = 0

    @staticmethod
    def supported(group=None) -> bool:
        """Single node, CUDA, every pair of devices peer-capable."""
        if not (torch.cuda.is_available() and dist.is_initialized()):
            return False
        world = dist.get_world_size(group)
        if world < 2:
            return False
        local = int(os.environ.get("LOCAL_WORLD_SIZE", str(world)))
        return local == world


class FusedDPAdamW:
    """Fused DP gradient reduction + AdamW over NVLink for a :class:`~meshy_b200.backend.flat.FlatParams`."""

    def __init__(self, flat, group=None, *, lr: float, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 0.0, max_norm: float = 1.0, timeout_s: float | None = None):
        self.flat = flat
        self.group = group
        self.lr = lr
        self.base_lr = lr
        self.betas = betas
        self.eps = eps
        self.weight_decay = weight_decay
        self.max_norm = max_norm
        self.step_count = 0
        self.mirror = None
        self.timeout_s = float(timeout_s if timeout_s is not None else os.environ.get("MESHY_SYMM_TIMEOUT_S", "30"))
        n = flat.numel
        dev = flat.master.device
        world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.world = world
        # equal shards, each a multiple of 4 elements (float4 accesses)
        per = -(-n // world)
        per = -(-per // 4) * 4
        self.lo = min(n, self.rank * per)
        self.hi = min(n, self.lo + per)
        n_pad = per * world
        sep = flat.separate_compute
        # with a bf16 compute copy the fp32 master is sharded like the moments: it stays a local buffer of
        # which only [lo, hi) is kept current, and only the bf16 copy is replicated (by the push); without
        # one the master itself is the replicated weight buffer and lives in the heap
        need = _align(n_pad * 4) * (1 if sep else 2) + (_align(n_pad * 2) if sep else 0) + 2 * _align(world * 4) \
            + 4096
        self.heap = SymmetricHeap(need, group, dev)
        self.master_tab = None
        if not sep:
            master, self.master_tab = self.heap.alloc(n_pad, torch.float32)
        grad, self.grad_tab = self.heap.alloc(n_pad, torch.float32)
        self.compute_tab = None
        if sep:
            compute, self.compute_tab = self.heap.alloc(n_pad, flat.compute.dtype)
        _, self.flag_tab = self.heap.alloc(world, torch.int32)
        _, self.slot_tab = self.heap.alloc(world, torch.float32)
        with torch.no_grad():
            grad[:n].copy_(flat.grad)
            if sep:
                compute[:n].copy_(flat.compute)
            else:
                master[:n].copy_(flat.master)
        flat.grad = grad[:n]
        if sep:
            flat.compute = compute[:n]
            flat.master_shard = (self.lo, self.hi, group, per)
        else:
            flat.master = master[:n]
            flat.compute = flat.master
        for s, p in zip(flat.slots, flat.params):
            p.data = flat.compute[s.offset:s.offset + s.numel].view(s.shape)
            g = flat.grad[s.offset:s.offset + s.numel].view(s.shape)
            if sep:
                p.main_grad = g
            else:
                p.grad = g
        # ZeRO-1: each rank keeps the AdamW moments of its shard only (2 x 4 bytes x n / world)
        shard = self.hi - self.lo
        for name in ("exp_avg", "exp_avg_sq"):
            full = getattr(flat, name)
            part = torch.zeros(shard, dtype=torch.float32, device=dev)
            if full is not None:
                part.copy_(full[self.lo:self.hi])
            setattr(flat, name, part)
        flat.moment_range = (self.lo, self.hi)
        self.scalars = torch.zeros(2, dtype=torch.float32, device=dev)
        self.epoch = 0
        dist.barrier(group)

    def step(self, grad_norm=None) -> torch.Tensor:
        """All ranks call this together after backward; returns the global gradient norm (device scalar)."""
        f = self.flat
        self.step_count += 1
        b1, b2 = self.betas
        self.epoch += 3
        ext().symm_dp_adamw(self.grad_tab, self.master_tab, self.compute_tab, self.flag_tab, self.slot_tab, f.master,
                            f.grad, f.exp_avg, f.exp_avg_sq, self.scalars, self.rank, self.world, self.lo, self.hi,
                            self.epoch, float(self.max_norm), float(self.lr), float(b1), float(b2), float(self.eps),
                            float(self.weight_decay), int(self.step_count), self.timeout_s)
        if self.mirror is not None:
            self.mirror.copy_(f.compute if f.separate_compute else f.master)
        # a copy: the scalar buffer is rewritten by the next step, and callers keep the norms of several steps
        return self.scalars[1].clone()

    def check(self) -> None:
        """Raise if a bounded wait of the step timed out (reads the device error word: a host sync)."""
        err = int(ext().device_error())
        if err:
            raise RuntimeError(f"fused DP step failed on rank {self.rank}: device error code {err} "
                               "(a peer did not arrive within the wait limit)")

    def full_moments(self) -> tuple[torch.Tensor, torch.Tensor]:
        """All-gather the sharded moments into full-length tensors (collective; checkpoints only)."""
        f = self.flat
        per = -(-f.numel // self.world)
        per = -(-per // 4) * 4
        out = []
        for buf in (f.exp_avg, f.exp_avg_sq):
            mine = torch.zeros(per, dtype=buf.dtype, device=buf.device)
            mine[:buf.numel()].copy_(buf)
            parts = [torch.empty_like(mine) for _ in range(self.world)]
            dist.all_gather(parts, mine, group=self.group)
            out.append(torch.cat(parts)[:f.numel])
        return out[0], out[1]

    def set_full_moments(self, exp_avg: torch.Tensor, exp_avg_sq: torch.Tensor) -> None:
        """Keep this rank's shard of full-length moments (after loading a checkpoint)."""
        self.flat.exp_avg.copy_(exp_avg.reshape(-1)[self.lo:self.hi])
        self.flat.exp_avg_sq.copy_(exp_avg_sq.reshape(-1)[self.lo:self.hi])

    def state_dict(self) -> dict:
        m, v = self.full_moments()
        return {"step": self.step_count, "exp_avg": m, "exp_avg_sq": v, "lr": self.lr}

    def load_state_dict(self, sd: dict) -> None:
        self.step_count = int(sd["step"])
        self.set_full_moments(sd["exp_avg"].to(self.flat.exp_avg.device), sd["exp_avg_sq"].to(self.flat.exp_avg.device))
        self.lr = float(sd.get("lr", self.lr))


__all__ = ["FusedDPAdamW", "SymmetricHeap"]
