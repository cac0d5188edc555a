"""Fully sharded data parallelism over flat buffers (parameters, gradients and optimiser state sharded).

The reference shards every trainer through torchtitan's FSDP2 (``fully_shard`` per transformer block plus
the root module, ``TT:torchtitan/models/llama4/parallelize.py:170-240``, driven by ``dp_shard`` in
``meshy/config.py:83-146``). This module is the same idea laid out for this framework's flat buffers:

* **units**: every transformer block is one unit; the embedding, the final norm and the LM head form the
  root unit. A unit's parameters are packed like :class:`~meshy_b200.backend.flat.FlatParams` packs a model
  (named order, 128-byte aligned offsets), padded to ``world x shard`` elements;
* **shards**: rank ``r`` keeps elements ``[r * shard, (r + 1) * shard)`` of every unit in five flat shard
  buffers (fp32 master, fp32 gradient, both AdamW moments, and the compute-dtype copy), so
  :class:`~meshy_b200.backend.flat.FlatAdamW` steps the shards unchanged -- one fused kernel over
  ``1 / world`` of the model;
* **forward**: the root unit is gathered once per weight version into its own buffer; blocks use two
  gather buffers (block ``i`` always lives in buffer ``i % 2``, so parameter views never move). Block
  ``i + 1`` is gathered on a side stream while block ``i`` computes, after block ``i - 1`` (the previous
  user of that buffer) has finished;
* **backward**: an identity autograd node at each block's output re-gathers the block (prefetching the
  next one down) before its backward runs; one at its input fires once the block's gradients are complete
  and reduce-scatters the block's full-size fp32 gradient buffer into the gradient shard on the side
  stream (accumulating across micro-batches), then zeroes it for block ``i - 2``. The root unit is reduced
  when the trainer folds the gradients after backward (:meth:`ShardedFlat.collect_cpu_grads`);
* **HSDP**: with a replicate group, the gradient shards are all-reduced across it before the step (the
  trainer's gradient reducer runs over the replicate group on the shard buffer).

Collectives. On one node with peer-capable GPUs (the default there) the compute shards and the full-size
gradient buffers live in a symmetric heap (CUDA IPC, :class:`~meshy_b200.parallel.symm.SymmetricHeap`):
a gather is one kernel that reads every rank's shard over NVLink into the local full-size buffer, and a
reduce-scatter is one kernel that sums this rank's slice of every rank's gradient buffer into the local
gradient shard (``csrc/kernels/fsdp.cu``), bracketed by bounded device barriers; the first gather after an
optimiser step waits at a barrier for every rank's step. Elsewhere (and on the CPU, with gloo) they are
``all_gather_into_tensor`` / ``reduce_scatter_tensor``. A weight sync and a checkpoint read the full model
through :meth:`ShardedFlat.full_buffer`, which re-assembles the global flat layout -- the shard -> replica
reshard an inference engine needs.
"""

from __future__ import annotations

import contextlib
import os

import torch
import torch.distributed as dist
import torch.nn as nn

from ..backend.flat import ALIGN, Slot, _align
from ..ops._ext import ext
from ..ops.functional import native


class _Unit:
    def __init__(self, idx: int, names: list[str], params: list[nn.Parameter], world: int):
        self.idx = idx
        self.names = names
        self.params = params
        self.local = []  # (offset within the unit, numel, shape) per parameter
        off = 0
        for p in params:
            self.local.append((off, p.numel(), tuple(p.shape)))
            off += _align(p.numel())
        self.numel = off
        self.shard = max(ALIGN, -(-off // (world * ALIGN)) * ALIGN)
        self.shard_off = 0  # offset of this unit's shard in the local shard buffers
        self.full = self.shard * world


class BlockBoundary(torch.autograd.Function):
    """Identity whose backward tells ``engine`` (the sharding engine, or the data-parallel reducer) that a
    block's backward begins (``where="out"``) or ends (``where="in"``)."""

    @staticmethod
    def forward(ctx, x, engine, i, where):
        ctx.engine, ctx.i, ctx.where = engine, i, where
        return x.view_as(x)

    @staticmethod
    def backward(ctx, g):
        if ctx.where == "out":
            ctx.engine.backward_begin(ctx.i)
        else:
            ctx.engine.backward_end(ctx.i)
        return g, None, None, None


class ShardedFlat:
    """Sharded counterpart of :class:`~meshy_b200.backend.flat.FlatParams` (see the module docstring).

    ``master`` / ``grad`` / ``exp_avg`` / ``exp_avg_sq`` / ``compute`` are this rank's shards (length
    ``numel``); ``slots`` describe the GLOBAL flat layout (the one an inference engine's weight buffer uses),
    which :meth:`full_buffer` fills."""

    sharded = True

    def __init__(self, model: nn.Module, group, *, compute_dtype: torch.dtype, device, replicate_group=None):
        self.device = torch.device(device)
        self.compute_dtype = compute_dtype
        self.group = group
        self.replicate_group = replicate_group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.separate_compute = compute_dtype != torch.float32
        named = list(model.named_parameters())
        # global layout (FlatParams / flatten_module order)
        self.slots: list[Slot] = []
        self.params: list[nn.Parameter] = []
        off = 0
        for name, p in named:
            self.slots.append(Slot(name, off, p.numel(), tuple(p.shape)))
            self.params.append(p)
            off += _align(p.numel())
        self.global_numel = off
        self.n_real = sum(s.numel for s in self.slots)
        # units: blocks by index, the rest in the root unit
        blocks: dict[int, list] = {}
        root = []
        for name, p in named:
            parts = name.split(".")
            if parts[0] == "layers" and len(parts) > 2 and parts[1].isdigit():
                blocks.setdefault(int(parts[1]), []).append((name, p))
            else:
                root.append((name, p))
        self.n_blocks = len(blocks)
        assert sorted(blocks) == list(range(self.n_blocks)), "blocks must be numbered 0..L-1"
        self.root = _Unit(-1, [n for n, _ in root], [p for _, p in root], self.world)
        self.blocks = [_Unit(i, [n for n, _ in blocks[i]], [p for _, p in blocks[i]], self.world)
                       for i in range(self.n_blocks)]
        soff = 0
        for u in [self.root] + self.blocks:
            u.shard_off = soff
            soff += u.shard
        self.numel = soff
        dev = self.device
        f32 = torch.float32
        self.master = torch.zeros(self.numel, dtype=f32, device=dev)
        self.grad = torch.zeros(self.numel, dtype=f32, device=dev)
        self.exp_avg = torch.zeros(self.numel, dtype=f32, device=dev)
        self.exp_avg_sq = torch.zeros(self.numel, dtype=f32, device=dev)
        self.compute = torch.zeros(self.numel, dtype=compute_dtype, device=dev) if self.separate_compute \
            else self.master
        self.peer = self._peer_capable()
        self.heap = None
        self._alloc_full()
        # shards from the (identical on every rank) initial values; parameter views into the full buffers
        with torch.no_grad():
            for u in [self.root] + self.blocks:
                full = torch.zeros(u.full, dtype=f32, device=dev)
                for p, (o, n, _) in zip(u.params, u.local):
                    full[o:o + n].copy_(p.detach().reshape(-1).float())
                self.master[u.shard_off:u.shard_off + u.shard].copy_(full[self.rank * u.shard:(self.rank + 1) * u.shard])
            if self.separate_compute:
                self.compute.copy_(self.master)
        self._bind()
        self.version = 0           # bumped whenever the shards change (optimiser step, load)
        self._cuda = self.device.type == "cuda"
        self._side = torch.cuda.Stream(device=self.device) if self._cuda else None
        self._ev: dict = {}
        self.comm_bytes = 0

    # ------------------------------------------------------------------ layout
    def _peer_capable(self) -> bool:
        if self.device.type != "cuda" or not self.separate_compute or os.environ.get("MESHY_FSDP_PEER", "1") == "0":
            return False
        if not native(self.master) or dist.get_backend(self.group) != "nccl":
            return False
        from .symm import SymmetricHeap

        return SymmetricHeap.supported(self.group) and self.world <= 8

    def _alloc_full(self) -> None:
        """Full-size buffers: the root unit's weights and gradients, two blocks' worth of each. In peer mode the
        compute shard and the gradient buffers are carved from a symmetric heap (mapped by every rank)."""
        dev, f32 = self.device, torch.float32
        bmax = max((u.full for u in self.blocks), default=ALIGN)
        self.root_w = torch.zeros(self.root.full, dtype=self.compute_dtype, device=dev)
        self.block_w = [torch.zeros(bmax, dtype=self.compute_dtype, device=dev) for _ in range(2)]
        if self.peer:
            from .symm import SymmetricHeap

            if self.heap is None:
                nbytes = self.numel * 2 + (self.root.full + 2 * bmax) * 4 + 8 * 1024
                self.heap = SymmetricHeap(nbytes, self.group, dev)
                shard, self.t_compute = self.heap.alloc(self.numel, self.compute_dtype)
                self.root_g, self.t_root_g = self.heap.alloc(self.root.full, f32)
                g0, t0 = self.heap.alloc(bmax, f32)
                g1, t1 = self.heap.alloc(bmax, f32)
                self._heap_g = [g0, g1]
                self.t_block_g = [t0, t1]
                self._flags, self.t_flags = self.heap.alloc(self.world, torch.int32)
                self._flags.zero_()
                self._heap_compute = shard
                self.epoch = 0
                self.timeout_s = float(os.environ.get("MESHY_SYMM_TIMEOUT_S", "30"))
            self._heap_compute.copy_(self.compute)
            self.compute = self._heap_compute
            self.root_g.zero_()
            for g in self._heap_g:
                g.zero_()
            self.block_g = list(self._heap_g)
            torch.cuda.synchronize(dev)
            dist.barrier(group=self.group)  # every region is mapped and initialised everywhere
        else:
            self.root_g = torch.zeros(self.root.full, dtype=f32, device=dev)
            self.block_g = [torch.zeros(bmax, dtype=f32, device=dev) for _ in range(2)]
        self._rs_tmp = torch.zeros(max([u.shard for u in self.blocks] + [self.root.shard]), dtype=f32, device=dev)
        self._holder = [None, None]  # (block, version) held by each block buffer
        self._root_version = -1

    def _bind(self) -> None:
        """Point every parameter (and its fp32 main_grad) at its unit's full buffers."""
        for u in [self.root] + self.blocks:
            w = self.root_w if u.idx < 0 else self.block_w[u.idx % 2]
            g = self.root_g if u.idx < 0 else self.block_g[u.idx % 2]
            for p, (o, n, shape) in zip(u.params, u.local):
                p.data = w[o:o + n].view(shape)
                if self.separate_compute:
                    p.main_grad = g[o:o + n].view(shape)
                    p.requires_grad_(True)
                else:
                    p.grad = None

    def _shard(self, buf: torch.Tensor, u: _Unit) -> torch.Tensor:
        return buf[u.shard_off:u.shard_off + u.shard]

    # ------------------------------------------------------------------ events / streams
    def _record(self, key) -> None:
        if self._cuda:
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(self.device))
            self._ev[key] = ev

    def _side_ctx(self):
        return torch.cuda.stream(self._side) if self._cuda else contextlib.nullcontext()

    def _side_wait(self, key) -> None:
        ev = self._ev.get(key)
        if ev is not None:
            self._side.wait_event(ev)

    def _main_wait(self, key) -> None:
        ev = self._ev.get(key)
        if ev is not None:
            torch.cuda.current_stream(self.device).wait_event(ev)

    def _side_record(self, key) -> None:
        if self._cuda:
            ev = torch.cuda.Event()
            ev.record(self._side)
            self._ev[key] = ev

    # ------------------------------------------------------------------ collectives
    def _barrier(self) -> None:
        self.epoch += 1
        ext().symm_barrier(self.t_flags, self.rank, self.world, self.epoch, self.timeout_s)

    def _gather(self, u: _Unit, out: torch.Tensor) -> None:
        if self.peer:
            es = self.compute.element_size()
            ext().fsdp_gather(self.t_compute, u.shard_off * es, u.shard * es, out)
        else:
            shard = self._shard(self.compute, u)
            dist.all_gather_into_tensor(out[:u.full], shard, group=self.group)
        self.comm_bytes += u.full * out.element_size()

    def _reduce(self, u: _Unit, full: torch.Tensor, table=None) -> None:
        if self.peer:
            self._barrier()  # every rank's gradients of this unit are complete
            ext().fsdp_reduce(table, 0, u.shard, self.rank, self._shard(self.grad, u))
            self._barrier()  # every rank has read this rank's buffer
        else:
            tmp = self._rs_tmp[:u.shard]
            dist.reduce_scatter_tensor(tmp, full[:u.full], group=self.group)
            self._shard(self.grad, u).add_(tmp)
        full[:u.full].zero_()
        self.comm_bytes += u.full * 4

    # ------------------------------------------------------------------ forward hooks
    def begin_forward(self) -> None:
        if self._cuda:  # buffers may still be read by work queued before this forward
            self._side.wait_stream(torch.cuda.current_stream(self.device))
        if self._root_version != self.version:
            if self.peer:  # every rank has finished the step that rewrote its shards
                with self._side_ctx():
                    self._barrier()
            with self._side_ctx():
                self._gather(self.root, self.root_w)
            self._side_record(("root",))
            self._main_wait(("root",))
            self._root_version = self.version
        if self.n_blocks:
            self._fetch(0, after=("start",))

    def _fetch(self, i: int, after) -> None:
        """Gather block ``i`` into buffer ``i % 2`` on the side stream once event ``after`` (the last use of
        that buffer) has passed; without that event, once everything queued on the compute stream has."""
        b = i % 2
        if self._holder[b] == (i, self.version):
            return
        if self._cuda:
            if after in self._ev:
                self._side_wait(after)
            else:
                self._side.wait_stream(torch.cuda.current_stream(self.device))
        with self._side_ctx():
            self._gather(self.blocks[i], self.block_w[b])
        self._side_record(("w", i))
        self._holder[b] = (i, self.version)

    def pre_block(self, i: int, x: torch.Tensor) -> torch.Tensor:
        self._main_wait(("w", i))
        if i + 1 < self.n_blocks:
            self._fetch(i + 1, after=("fwd", i - 1))
        if torch.is_grad_enabled() and x.requires_grad:
            x = BlockBoundary.apply(x, self, i, "in")
        return x

    def post_block(self, i: int, x: torch.Tensor) -> torch.Tensor:
        self._record(("fwd", i))
        if torch.is_grad_enabled() and x.requires_grad:
            x = BlockBoundary.apply(x, self, i, "out")
        return x

    # ------------------------------------------------------------------ backward hooks
    def backward_begin(self, i: int) -> None:
        self._fetch(i, after=("bwd", i + 2))
        self._main_wait(("w", i))
        self._main_wait(("rs", i + 2))  # the gradient buffer this block accumulates into is free again
        if i >= 1:
            self._fetch(i - 1, after=("bwd", i + 1))

    def backward_end(self, i: int) -> None:
        u = self.blocks[i]
        self._fold(u, self.block_g[i % 2])
        self._record(("bwd", i))
        if self._cuda:
            self._side_wait(("bwd", i))
        with self._side_ctx():
            self._reduce(u, self.block_g[i % 2], self.t_block_g[i % 2] if self.peer else None)
        self._side_record(("rs", i))

    def _fold(self, u: _Unit, full: torch.Tensor) -> None:
        """PyTorch paths leave ``.grad`` tensors: add them to the unit's fp32 gradient buffer."""
        with torch.no_grad():
            for p, (o, n, _) in zip(u.params, u.local):
                if p.grad is not None:
                    full[o:o + n].add_(p.grad.reshape(-1).float())
                    p.grad = None

    def collect_cpu_grads(self) -> None:
        """Called by the trainer after every backward: reduce the root unit and wait for the side stream."""
        self._fold(self.root, self.root_g)
        if self._cuda:
            self._side.wait_stream(torch.cuda.current_stream(self.device))
        with self._side_ctx():
            self._reduce(self.root, self.root_g, self.t_root_g if self.peer else None)
        if self._cuda:
            torch.cuda.current_stream(self.device).wait_stream(self._side)
        self._ev.clear()

    # ------------------------------------------------------------------ optimiser interface
    def zero_grad(self) -> None:
        self.grad.zero_()

    def weights_changed(self) -> None:
        self.version += 1

    def grad_norm(self) -> torch.Tensor:
        if self.grad.is_cuda and native(self.grad):
            out = torch.zeros(1, dtype=torch.float32, device=self.device)
            ext().sq_norm(self.grad, out)
        else:
            out = (self.grad.double() ** 2).sum().float().reshape(1)
        dist.all_reduce(out, group=self.group)
        return out.sqrt().reshape(())

    def recast(self) -> None:
        if self.separate_compute:
            self.compute.copy_(self.master)
        self.weights_changed()

    def shard_views(self, buf: torch.Tensor, names) -> list[torch.Tensor]:
        """This rank's pieces of the named parameters inside a shard buffer."""
        wanted = set(names)
        out = []
        for u in [self.root] + self.blocks:
            lo_r, hi_r = self.rank * u.shard, (self.rank + 1) * u.shard
            for name, (o, n, _) in zip(u.names, u.local):
                if name not in wanted:
                    continue
                lo, hi = max(o, lo_r), min(o + n, hi_r)
                if lo < hi:
                    out.append(buf[u.shard_off + lo - lo_r:u.shard_off + hi - lo_r])
        return out

    # ------------------------------------------------------------------ full views (collectives)
    def full_buffer(self, which: str = "compute", out: torch.Tensor | None = None) -> torch.Tensor:
        """Re-assemble shard buffer ``which`` into the global flat layout (every rank of the shard group must
        call this)."""
        src = getattr(self, which)
        dtype = src.dtype
        if out is None:
            out = torch.zeros(self.global_numel, dtype=dtype, device=self.device)
        by_name = {s.name: s for s in self.slots}
        for u in [self.root] + self.blocks:
            full = torch.empty(u.full, dtype=dtype, device=self.device)
            dist.all_gather_into_tensor(full, self._shard(src, u).contiguous(), group=self.group)
            for name, (o, n, _) in zip(u.names, u.local):
                s = by_name[name]
                out[s.offset:s.offset + n].copy_(full[o:o + n])
        return out

    def set_full(self, which: str, full: torch.Tensor) -> None:
        """Take this rank's shard of a global-layout buffer into shard buffer ``which``."""
        dst = getattr(self, which)
        by_name = {s.name: s for s in self.slots}
        with torch.no_grad():
            for u in [self.root] + self.blocks:
                unit = torch.zeros(u.full, dtype=dst.dtype, device=dst.device)
                for name, (o, n, _) in zip(u.names, u.local):
                    s = by_name[name]
                    unit[o:o + n].copy_(full[s.offset:s.offset + n])
                self._shard(dst, u).copy_(unit[self.rank * u.shard:(self.rank + 1) * u.shard])

    def gather_master(self) -> None:  # the checkpoint path reads full buffers instead
        return None

    def state_dict(self, source: str = "master") -> dict[str, torch.Tensor]:
        buf = self.full_buffer("master" if source == "master" else "compute")
        return {s.name: buf[s.offset:s.offset + s.numel].view(s.shape) for s in self.slots}

    def load_state_dict(self, sd: dict[str, torch.Tensor]) -> None:
        full = torch.zeros(self.global_numel, dtype=torch.float32, device=self.device)
        for s in self.slots:
            full[s.offset:s.offset + s.numel].copy_(sd[s.name].reshape(-1).float())
        self.set_full("master", full)
        self.recast()

    def check(self) -> None:
        """Raise if a bounded device wait of the peer collectives timed out (reads the device error word)."""
        err = int(ext().device_error()) if self.peer else 0
        if err:
            raise RuntimeError(f"sharded-parameter collective failed on rank {self.rank}: device error code {err}")

    def close(self) -> None:
        if self.heap is not None:
            torch.cuda.synchronize(self.device)
            self.heap.close()
            self.heap = None

    # ------------------------------------------------------------------ colocation hand-off
    _SHARDS = ("master", "grad", "exp_avg", "exp_avg_sq", "compute")

    def offload(self) -> None:
        """Shards to pinned host memory; the full-size buffers are dropped (they are re-gathered)."""
        if self.master is None or self.device.type != "cuda":
            return
        host = {}
        for name in self._SHARDS:
            if name == "compute" and (not self.separate_compute or self.peer):  # heap memory stays mapped
                continue
            t = getattr(self, name)
            h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
            h.copy_(t, non_blocking=True)
            host[name] = h
        torch.cuda.synchronize()
        self._host = host
        for name in host:
            setattr(self, name, None)
        if not self.separate_compute:
            self.compute = None
        self.root_w = self._rs_tmp = None
        self.block_w = [None, None]
        if not self.peer:
            self.root_g = None
            self.block_g = [None, None]
        for p in self.params:
            p.data = torch.empty(0, dtype=p.dtype, device=p.device)
            p.main_grad = None
        self._ev.clear()
        torch.cuda.empty_cache()

    def restore(self) -> None:
        host = getattr(self, "_host", None)
        if not host:
            return
        for name, h in host.items():
            setattr(self, name, h.to(self.device, non_blocking=True))
        if not self.separate_compute:
            self.compute = self.master
        self._alloc_full()
        self._bind()
        torch.cuda.synchronize()
        self._host = None

    @property
    def sync_source(self) -> torch.Tensor:
        """Full compute-dtype weights in the global layout (gathered; a collective over the shard group)."""
        return self.full_buffer("compute" if self.separate_compute else "master")


__all__ = ["ShardedFlat"]
