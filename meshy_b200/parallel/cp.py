"""Context parallelism: head-tail sequence sharding and attention over the gathered sequence.

Reference behaviour (``meshy/backend/titan/cp.py:42-162``, torchtitan ``cp_shard``
and torch's CP SDPA dispatcher with its default all-gather rotation):

* a ``[rows, S]`` block is split into ``2 * cp`` chunks of ``c = S / (2 cp)``
  tokens; CP rank ``r`` keeps chunks ``r`` and ``2 cp - 1 - r`` (head-tail /
  zig-zag), which gives every rank the same amount of causal attention work;
* :meth:`CpSharder.gather_seq` all-gathers the shards and restores temporal
  order (GAE and the critic need whole rows);
* per-document token counts are computed on the host from full samples here,
  so the reference's CP all-reduce of those counts is not needed
  (:meth:`CpSharder.all_reduce_sum` remains for callers that have sharded sums).

Attention, gathered path: each layer all-gathers K and V over the CP group
(the reference's rotation), reorders them into sequence order, and runs the
chunked causal kernel: the two local query chunks of a row are two query
documents at key positions ``r c`` and ``(2 cp - 1 - r) c`` of the gathered row
(:func:`meshy_b200.ops.functional.flash_attn_chunks`).  Backward reduce-scatters
dK / dV back to their owners.  The collectives go through NCCL (gloo on CPU).

Attention, peer path (opt-in, ``MESHY_CP_PEER=1``; one node, NCCL, head_dim
128, chunks a multiple of 128 tokens): the forward runs no all-gather. Every
rank copies its local K / V into a symmetric-memory buffer that every rank
maps, and the tcgen05 attention kernel reads each key tile straight from its
owner's buffer over NVLink with plain TMA loads (``_C.flash_attn_fwd_cp_peer``).
Two device barriers over the CP group bracket the copy (previous readers done;
every rank's K / V in place). The backward gathers K / V (NCCL), runs the
chunked backward kernels and reduce-scatters dK / dV, as the gathered path
does. It is off by default because it measured slower (B200, 2 ranks, 1 row,
12 query / 2 KV heads: forward 3.7 ms vs 0.8 ms at 16k tokens, 40.6 ms vs
7.7 ms at 64k): every (query block, head) CTA re-reads its key tiles, which a
local gathered buffer serves from L2, while peer reads cross NVLink each time.
"""

from __future__ import annotations

from contextlib import contextmanager
from dataclasses import dataclass

import torch
import torch.distributed as dist

from ..ops import functional as Fx


def _peer_enabled() -> bool:
    import os

    return os.environ.get("MESHY_CP_PEER", "0") == "1" and os.environ.get("MESHY_FA_TC", "1") != "0"


def _nccl(group) -> bool:
    return dist.get_backend(group) == "nccl"


class _AllGather(torch.autograd.Function):
    """``x [N, ...]`` → ``[cp * N, ...]`` (rank-major); backward sums the gradient slices back."""

    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        world = dist.get_world_size(group)
        x = x.contiguous()
        if _nccl(group):
            out = x.new_empty((world * x.shape[0],) + tuple(x.shape[1:]))
            dist.all_gather_into_tensor(out, x, group=group)
            return out
        parts = [torch.empty_like(x) for _ in range(world)]
        dist.all_gather(parts, x, group=group)
        return torch.cat(parts)

    @staticmethod
    def backward(ctx, g):
        group = ctx.group
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        g = g.contiguous()
        n = g.shape[0] // world
        if _nccl(group):
            out = g.new_empty((n,) + tuple(g.shape[1:]))
            dist.reduce_scatter_tensor(out, g, group=group)
            return out, None
        g = g.clone()
        dist.all_reduce(g, group=group)
        return g[rank * n:(rank + 1) * n], None


@dataclass
class CpLayout:
    rows: int
    seq_len: int   # S (global, per row)
    chunk: int     # c = S / (2 cp)


class _CpPeerAttn(torch.autograd.Function):
    """Forward: K / V read in place on every CP rank (no all-gather). Backward: the gathered path."""

    @staticmethod
    def forward(ctx, q, k, v, sharder, layout, scale):
        out, lse = sharder._peer_forward(q, k, v, layout, scale)
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.sharder, ctx.layout, ctx.scale = sharder, layout, scale
        return out

    @staticmethod
    def backward(ctx, g):
        q, k, v, out, lse = ctx.saved_tensors
        gq, gk, gv = ctx.sharder._gathered_backward(q, k, v, out, lse, g.contiguous(), ctx.layout, ctx.scale)
        return gq, gk, gv, None, None, None


class CpSharder:
    def __init__(self, group):
        self.group = group
        self.size = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self._heap = None       # symmetric K / V buffers of the peer path
        self._epoch = 0

    # ------------------------------------------------------------------ index maps
    def chunk_ids(self, rank: int | None = None) -> tuple[int, int]:
        r = self.rank if rank is None else rank
        return r, 2 * self.size - 1 - r

    def local_index(self, S: int, device=None) -> torch.Tensor:
        """Positions (within a row of ``S``) this rank keeps, in local order."""
        c = S // (2 * self.size)
        a, b = self.chunk_ids()
        return torch.cat([torch.arange(a * c, (a + 1) * c, device=device), torch.arange(b * c, (b + 1) * c, device=device)])

    def gather_order(self, S: int, device=None) -> torch.Tensor:
        """Index into the rank-major concatenation of every rank's local row that yields sequence order."""
        c = S // (2 * self.size)
        pos = torch.empty(S, dtype=torch.long, device=device)
        for r in range(self.size):
            a, b = self.chunk_ids(r)
            base = r * 2 * c
            pos[a * c:(a + 1) * c] = torch.arange(base, base + c, device=device)
            pos[b * c:(b + 1) * c] = torch.arange(base + c, base + 2 * c, device=device)
        return pos

    # ------------------------------------------------------------------ tensors
    def shard_seq(self, *tensors: torch.Tensor) -> tuple[torch.Tensor, ...]:
        out = []
        for t in tensors:
            S = t.shape[1]
            if S % (2 * self.size):
                raise ValueError(f"sequence length {S} is not divisible by 2 x cp = {2 * self.size}")
            out.append(t.index_select(1, self.local_index(S, t.device)).contiguous())
        return tuple(out)

    def gather_seq(self, *tensors: torch.Tensor) -> tuple[torch.Tensor, ...]:
        out = []
        for t in tensors:
            rows, L = t.shape[:2]
            S = L * self.size
            full = _AllGather.apply(t.transpose(0, 1).contiguous(), self.group)  # [cp * L, rows, ...]
            out.append(full.index_select(0, self.gather_order(S, t.device)).transpose(0, 1).contiguous())
        return tuple(out)

    def all_reduce_sum(self, t: torch.Tensor) -> torch.Tensor:
        y = t.clone()
        dist.all_reduce(y, group=self.group)
        return y

    # ------------------------------------------------------------------ trainer batches
    def shard_batch(self, b):
        """Padded-layout :class:`~meshy_b200.backend.batch.Batch` → this rank's head-tail shard."""
        if b.layout != "padded":
            raise ValueError("context parallelism needs the padded batch layout (varlen + CP is not supported)")
        rows = b.rows
        S = b.n_tokens // rows
        idx = self.local_index(S, b.input_ids.device)

        def sh(t):
            if t is None or t.dim() == 0 or t.shape[0] != rows * S:
                return t
            return t.view(rows, S, *t.shape[1:]).index_select(1, idx).reshape(rows * idx.numel(), *t.shape[1:])

        L = idx.numel()
        b.input_ids, b.labels, b.positions, b.mask, b.doc_ids = (sh(b.input_ids), sh(b.labels), sh(b.positions),
                                                                 sh(b.mask), sh(b.doc_ids))
        if b.adv_per_token:
            b.advantages = sh(b.advantages)
        b.rollout_logprobs = sh(b.rollout_logprobs)
        b.cu_seqlens = torch.arange(0, rows * L + 1, L, dtype=torch.int32, device=b.input_ids.device)
        b.max_seqlen = L
        b.extra["cp"] = CpLayout(rows, S, S // (2 * self.size))
        return b

    # ------------------------------------------------------------------ attention
    def peer_ok(self, q, layout: CpLayout) -> bool:
        """Whether the no-all-gather peer path applies to this call."""
        if not (q.is_cuda and _peer_enabled() and _nccl(self.group) and self.size <= 8):
            return False
        from .symm import SymmetricHeap

        return q.shape[-1] == 128 and layout.chunk % 128 == 0 and SymmetricHeap.supported(self.group)

    def _barrier(self) -> None:
        from ..ops._ext import ext

        self._epoch += 1
        ext().symm_barrier(self._flags, self.rank, self.size, self._epoch, 30.0)

    def _peer_buffers(self, numel: int):
        """Symmetric K and V buffers of at least ``numel`` bf16 elements (collective on first use / growth)."""
        from .symm import SymmetricHeap

        if self._heap is None or self._cap < numel:
            if self._heap is not None:
                torch.cuda.synchronize()
                dist.barrier(self.group)
                self._heap.close()
            cap = max(numel, 1 << 20)
            self._heap = SymmetricHeap(2 * cap * 2 + 4096, self.group)
            self._kbuf, ktab = self._heap.alloc(cap, torch.bfloat16)
            self._vbuf, vtab = self._heap.alloc(cap, torch.bfloat16)
            _, self._flags = self._heap.alloc(self.size, torch.int32)
            self._kptrs, self._vptrs = ktab.tolist(), vtab.tolist()
            self._cap, self._epoch = cap, 0
            dist.barrier(self.group)
        return self._kbuf, self._vbuf

    def close(self) -> None:
        if self._heap is not None:
            torch.cuda.synchronize()
            dist.barrier(self.group)
            self._heap.close()
            self._heap = None

    def _peer_forward(self, q, k, v, layout: CpLayout, scale: float):
        from ..ops._ext import ext

        rows, c = layout.rows, layout.chunk
        n = k.numel()
        kb, vb = self._peer_buffers(n)
        self._barrier()  # every rank has finished reading the previous contents
        kb[:n].copy_(k.reshape(-1))
        vb[:n].copy_(v.reshape(-1))
        self._barrier()  # every rank's K / V are in place
        dev = q.device
        a, b = self.chunk_ids()
        cu_q = torch.arange(0, rows * 2 * c + 1, c, dtype=torch.int32, device=dev)
        q_off = torch.tensor([a * c, b * c], dtype=torch.int32, device=dev).repeat(rows)
        out = torch.empty_like(q)
        lse = torch.empty(q.shape[1], q.shape[0], dtype=torch.float32, device=dev)
        ext().flash_attn_fwd_cp_peer(q.contiguous(), self._kptrs, self._vptrs, rows, c, k.shape[1], cu_q, q_off, 2,
                                     out, lse, c, float(scale))
        return out, lse

    def _gathered_kv(self, k, v, layout: CpLayout):
        """K / V of the whole rows in sequence order (differentiable: backward reduce-scatters)."""
        rows, S, c = layout.rows, layout.seq_len, layout.chunk
        dev = k.device
        kf = _AllGather.apply(k, self.group)  # [cp * rows * 2c, Hkv, hd], rank-major
        vf = _AllGather.apply(v, self.group)
        # rank-major [cp, rows, 2c] → [rows, S] in sequence order
        order = self.gather_order(S, dev)
        rank_of = order // (2 * c)
        within = order % (2 * c)
        src = (rank_of.unsqueeze(0) * rows * 2 * c + torch.arange(rows, device=dev).unsqueeze(1) * 2 * c
               + within.unsqueeze(0)).reshape(-1)
        return kf.index_select(0, src), vf.index_select(0, src)

    def _gathered_backward(self, q, k, v, out, lse, g, layout: CpLayout, scale: float):
        from ..ops._ext import ext

        rows, S, c = layout.rows, layout.seq_len, layout.chunk
        dev = q.device
        with torch.enable_grad():
            kd = k.detach().requires_grad_(True)
            vd = v.detach().requires_grad_(True)
            kf, vf = self._gathered_kv(kd, vd, layout)
        H, hd = q.shape[1], q.shape[2]
        qv, ov, gvw = q.view(rows, 2, c, H, hd), out.view(rows, 2, c, H, hd), g.view(rows, 2, c, H, hd)
        lv = lse.view(H, rows, 2, c)
        gq = torch.empty_like(q).view(rows, 2, c, H, hd)
        cu_q = torch.arange(0, rows * c + 1, c, dtype=torch.int32, device=dev)
        cu_k = torch.arange(0, rows * S + 1, S, dtype=torch.int32, device=dev)
        gkf = gvf = None
        kfd, vfd = kf.detach(), vf.detach()
        for j, chunk in enumerate(self.chunk_ids()):
            qj = qv[:, j].reshape(rows * c, H, hd).contiguous()
            oj = ov[:, j].reshape(rows * c, H, hd).contiguous()
            gj = gvw[:, j].reshape(rows * c, H, hd).contiguous()
            lj = lv[:, :, j].reshape(H, rows * c).contiguous()
            off = torch.full((rows,), chunk * c, dtype=torch.int32, device=dev)
            gqj, gkj, gvj = torch.empty_like(qj), torch.zeros_like(kfd), torch.zeros_like(vfd)
            ext().flash_attn_bwd_kv(qj, kfd, vfd, cu_q, cu_k, off, oj, gj, lj, gqj, gkj, gvj, c, S, float(scale))
            gq[:, j] = gqj.view(rows, c, H, hd)
            gkf = gkj if gkf is None else gkf + gkj
            gvf = gvj if gvf is None else gvf + gvj
        gk, gv = torch.autograd.grad((kf, vf), (kd, vd), (gkf, gvf))
        return gq.view_as(q), gk, gv

    def attention(self, q, k, v, layout: CpLayout, scale: float | None = None):
        """Local ``q/k/v [rows * 2c, H, hd]`` → local attention output, exact causal over full rows."""
        if scale is None:
            scale = 1.0 / (q.shape[-1] ** 0.5)
        if self.peer_ok(q, layout):
            return _CpPeerAttn.apply(q, k.contiguous(), v.contiguous(), self, layout, float(scale))
        rows, S, c = layout.rows, layout.seq_len, layout.chunk
        dev = q.device
        kf, vf = self._gathered_kv(k, v, layout)
        a, b = self.chunk_ids()
        H, hd = q.shape[1], q.shape[2]
        qv = q.view(rows, 2, c, H, hd)
        cu_q = torch.arange(0, rows * c + 1, c, dtype=torch.int32, device=dev)
        cu_k = torch.arange(0, rows * S + 1, S, dtype=torch.int32, device=dev)
        outs = []
        # the head chunk and the tail chunk of every row are two calls, so no key row is shared by two
        # query documents of one call (dK / dV of the two calls are summed by autograd)
        for j, chunk in enumerate((a, b)):
            qj = qv[:, j].reshape(rows * c, H, hd)
            off = torch.full((rows,), chunk * c, dtype=torch.int32, device=dev)
            outs.append(Fx.flash_attn_chunks(qj, kf, vf, cu_q, cu_k, off, c, S, scale).view(rows, 1, c, H, hd))
        return torch.cat(outs, 1).reshape(rows * 2 * c, H, hd)


@contextmanager
def cp_attention(sharder: CpSharder, layout: CpLayout):
    """Route the model's attention calls through ``sharder.attention`` for one forward/backward."""
    def attn(q, k, v, cu_seqlens, max_seqlen, scale=None):
        return sharder.attention(q, k, v, layout, scale)

    with Fx.attention_override(attn):
        yield


__all__ = ["CpLayout", "CpSharder", "cp_attention"]
