"""Expert parallelism: experts sharded over an EP group, tokens sent to their owners.

Expert ``e`` lives on EP rank ``e // E_local`` (``E_local = n_experts / ep``),
the layout torchtitan's ``ExpertParallel`` uses (experts sharded on dim 0,
``TT:torchtitan/distributed/expert_parallel.py:50-75``). One MoE layer:

1. route (top-k of the softmax router) on the local tokens;
2. **dispatch**: every (token, expert) assignment goes to the expert's owner;
3. the owner runs its local experts over what it received (grouped GEMMs);
4. **combine**: outputs go back and are summed at the source with the
   routing weights.

Two transports:

* **peer memory** (CUDA, one node; the default there): :class:`PeerExchange`.
  A source writes its token rows straight into the owner's receive regions
  with P2P stores from a kernel (``_C.ep_dispatch``), a bounded device barrier
  closes the exchange, the owner plans and gathers its local experts' rows on
  the device and runs the grouped tcgen05 GEMMs on its own memory, and a
  second kernel stores the expert outputs back into the sources' buffers
  (``_C.ep_return``). Backward runs the same exchanges for the gradients. No
  split sizes go through the host, and no TMA touches peer memory;
* **collective** (gloo on CPU, or several nodes): two ``all_to_all_single``
  calls with split sizes exchanged first, differentiable by running the
  inverse exchange in backward.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


class _AllToAll(torch.autograd.Function):
    """``all_to_all_single`` with uneven splits; backward sends gradients the opposite way."""

    @staticmethod
    def forward(ctx, x, send_splits: list[int], recv_splits: list[int], group):
        ctx.group, ctx.send, ctx.recv = group, send_splits, recv_splits
        out = x.new_empty((sum(recv_splits),) + tuple(x.shape[1:]))
        dist.all_to_all_single(out, x.contiguous(), recv_splits, send_splits, group=group)
        return out

    @staticmethod
    def backward(ctx, g):
        out = g.new_empty((sum(ctx.send),) + tuple(g.shape[1:]))
        dist.all_to_all_single(out, g.contiguous(), ctx.send, ctx.recv, group=ctx.group)
        return out, None, None, None


def all_to_all(x: torch.Tensor, send_splits: list[int], recv_splits: list[int], group) -> torch.Tensor:
    return _AllToAll.apply(x, send_splits, recv_splits, group)


def _exchange_splits(send: torch.Tensor, group) -> list[int]:
    recv = torch.empty_like(send)
    dev = send.device
    if dist.get_backend(group) != "nccl":
        send, recv = send.cpu(), recv.cpu()
    dist.all_to_all_single(recv, send, group=group)
    return recv.to(dev).tolist()


class PeerExchange:
    """Symmetric receive regions of one EP group, shared by every MoE layer of the model (layers run one
    after another, and each exchange ends with a device barrier before the next one can start).

    ``cap`` bounds the assignments (tokens x top-k) one rank sends per layer call; it is fixed when the
    regions are allocated (a collective, at trainer set-up)."""

    def __init__(self, group, dim: int, cap: int, device, timeout_s: float = 30.0):
        from .symm import SymmetricHeap

        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.dim, self.cap = int(dim), int(cap)
        self.timeout_s = timeout_s
        W, cap, D = self.world, self.cap, self.dim
        nbytes = W * cap * D * 2 + 2 * W * cap * 4 + cap * D * 2 + 2 * W * 4 + 16 * 256
        self.heap = SymmetricHeap(nbytes, group, device)
        self.recv_x, self.t_recv_x = self.heap.alloc(W * cap * D, torch.bfloat16)
        self.recv_meta, self.t_recv_meta = self.heap.alloc(W * cap, torch.int32)
        self.recv_idx, self.t_recv_idx = self.heap.alloc(W * cap, torch.int32)
        self.recv_cnt, self.t_recv_cnt = self.heap.alloc(W, torch.int32)
        self.ret, self.t_ret = self.heap.alloc(cap * D, torch.bfloat16)
        self.flags, self.t_flags = self.heap.alloc(W, torch.int32)
        self.recv_x = self.recv_x.view(W * cap, D)
        self.ret = self.ret.view(cap, D)
        self.epoch = 0
        dist.barrier(group=group)  # every region is mapped everywhere before anyone writes

    def barrier(self) -> None:
        self.epoch += 1
        ext().symm_barrier(self.t_flags, self.rank, self.world, self.epoch, self.timeout_s)

    def owner_plan(self, experts: torch.Tensor, e_local: int):
        """Stable placement of this rank's assignments per owner rank (the device plan over owner ids)."""
        n = experts.numel()
        owners = (experts.reshape(-1) // e_local).to(torch.int32)
        cnt = torch.empty(self.world, dtype=torch.int32, device=experts.device)
        off = torch.empty(self.world + 1, dtype=torch.int32, device=experts.device)
        slot = torch.empty(n, dtype=torch.int32, device=experts.device)
        row_src = torch.empty(_plan_rows(n, self.world), dtype=torch.int32, device=experts.device)
        ext().moe_plan(owners.reshape(-1, 1), cnt, off, slot, row_src, None, None)
        return slot, off, cnt

    def close(self) -> None:
        self.heap.close()


def _plan_rows(n: int, groups: int) -> int:
    from ..ops.moe import plan_rows

    return plan_rows(n, groups)


def ext():
    from ..ops._ext import ext as _e

    return _e()


# ─── the three phases of each direction (source → owner → source), between device barriers ───────────
# They are separate functions so one process can also play every rank in turn against local regions (the
# kernels only read and store through address tables; nothing in them waits on another rank).

def _fwd_dispatch(x, experts, xch, E_local):
    """Source: plan this rank's assignments per owner and store the token rows into the owners' regions."""
    k = experts.shape[1]
    ex = experts.reshape(-1).contiguous()
    slot_o, off_o, cnt_o = xch.owner_plan(ex, E_local)
    ext().ep_dispatch(x.contiguous(), k, ex, slot_o, off_o, cnt_o, E_local, xch.rank, xch.world, xch.cap,
                      xch.t_recv_x, xch.t_recv_meta, xch.t_recv_idx, xch.t_recv_cnt)
    return ex, slot_o, off_o, cnt_o


def _fwd_owner(xch, w13, w2):
    """Owner: local plan over everything received, grouped GEMMs on local memory, rows stored back to their
    sources' return regions."""
    from ..ops import moe as M

    C = ext()
    W, cap = xch.world, xch.cap
    E_local, F2 = w13.shape[0], w13.shape[1]
    D = xch.dim
    dev, dt = xch.recv_x.device, xch.recv_x.dtype
    ids = torch.empty(W * cap, dtype=torch.int32, device=dev)
    C.ep_recv_ids(xch.recv_meta, xch.recv_cnt, W, cap, E_local, ids)
    rows = M.plan_rows(W * cap, E_local)
    cnt = torch.empty(E_local, dtype=torch.int32, device=dev)
    off = torch.empty(E_local + 1, dtype=torch.int32, device=dev)
    slot = torch.empty(W * cap, dtype=torch.int32, device=dev)
    row_src = torch.empty(rows, dtype=torch.int32, device=dev)
    xp = torch.empty(rows, D, dtype=dt, device=dev)
    C.moe_plan(ids.view(-1, 1), cnt, off, slot, row_src, xch.recv_x, xp)
    idx = xch.recv_idx.clone()
    h = torch.empty(rows, F2, dtype=dt, device=dev)
    act = torch.empty(rows, F2 // 2, dtype=dt, device=dev)
    C.gemm_grouped(xp, w13, act, off, M.GRP_M, False, M.EPI_SWIGLU, h)
    y = torch.empty(rows, D, dtype=dt, device=dev)
    C.gemm_grouped(act, w2, y, off, M.GRP_M, False, M.EPI_STORE, None)
    C.ep_return(y, ids, slot, idx, W, cap, xch.cap, xch.t_ret)
    return ids, slot, off, cnt, row_src, idx, xp, h, act


def _fwd_collect(xch, n, weights, T):
    """Source: weighted sum of the returned rows (assignment i came back to ret[i])."""
    y_src = xch.ret[:n].clone()
    ident = torch.arange(n, dtype=torch.int32, device=y_src.device)
    out = torch.empty(T, xch.dim, dtype=y_src.dtype, device=y_src.device)
    ext().moe_combine(y_src, ident, weights.contiguous(), out)
    return out, y_src, ident


def _bwd_dispatch(dout, y_src, ident, weights, ex, slot_o, off_o, cnt_o, E_local, xch):
    """Source: gradients of the returned rows and of the routing weights; the row gradients go to the owners."""
    T, D = dout.shape
    n = ident.numel()
    dret = torch.empty(n, D, dtype=dout.dtype, device=dout.device)
    dw = torch.empty(T, n // T, dtype=torch.float32, device=dout.device)
    ext().moe_combine_bwd(dout.contiguous(), y_src, ident, weights, dret, dw)
    ext().ep_dispatch(dret, 1, ex, slot_o, off_o, cnt_o, E_local, xch.rank, xch.world, xch.cap, xch.t_recv_x,
                      None, None, None)
    return dw


def _bwd_owner(xch, ids, slot, off, row_src, idx, xp, h, act, w13, w2, block):
    """Owner: the experts' backward on its rows (weight gradients into main_grad when there is one); the input
    row gradients are stored back to their sources."""
    from ..ops import moe as M

    C = ext()
    W, cap = xch.world, xch.cap
    E_local, F2 = w13.shape[0], w13.shape[1]
    D = xch.dim
    rows = xp.shape[0]
    dev, dt = xp.device, xp.dtype
    dy = torch.empty(rows, D, dtype=dt, device=dev)
    C.gather_rows(row_src, off, xch.recv_x, dy)
    dact = torch.empty(rows, F2 // 2, dtype=dt, device=dev)
    C.gemm_grouped(dy, w2, dact, off, M.GRP_M, True, M.EPI_STORE, None)
    g2 = w2.main_grad if getattr(w2, "main_grad", None) is not None else torch.zeros(
        w2.shape, dtype=torch.float32, device=dev)
    C.gemm_grouped(dy, act, g2.view(E_local * D, F2 // 2), off, M.GRP_K, True, M.EPI_STORE, None)
    dh = torch.empty_like(h)
    C.swiglu_bwd(h, dact, dh, block)
    dxp = torch.empty(rows, D, dtype=dt, device=dev)
    C.gemm_grouped(dh, w13, dxp, off, M.GRP_M, True, M.EPI_STORE, None)
    g13 = w13.main_grad if getattr(w13, "main_grad", None) is not None else torch.zeros(
        w13.shape, dtype=torch.float32, device=dev)
    C.gemm_grouped(dh, xp, g13.view(E_local * F2, D), off, M.GRP_K, True, M.EPI_STORE, None)
    C.ep_return(dxp, ids, slot, idx, W, cap, xch.cap, xch.t_ret)
    return g13, g2


def _bwd_collect(xch, ident, T):
    """Source: token gradient = sum over its k returned rows."""
    n = ident.numel()
    dx = torch.empty(T, xch.dim, dtype=xch.ret.dtype, device=xch.ret.device)
    ext().moe_combine(xch.ret[:n].contiguous(), ident, None, dx)
    return dx


class _PeerExperts(torch.autograd.Function):
    """Expert-parallel routed-expert output over peer memory (see :class:`PeerExchange`)."""

    @staticmethod
    def forward(ctx, x, weights, experts, w13, w2, xch: PeerExchange, block: int):
        T = x.shape[0]
        n = T * experts.shape[1]
        if n > xch.cap:
            raise RuntimeError(f"expert-parallel layer got {n} assignments; the receive regions hold {xch.cap}")
        E_local = w13.shape[0]
        ex, slot_o, off_o, cnt_o = _fwd_dispatch(x, experts, xch, E_local)
        xch.barrier()
        ids, slot, off, cnt, row_src, idx, xp, h, act = _fwd_owner(xch, w13, w2)
        xch.barrier()
        out, y_src, ident = _fwd_collect(xch, n, weights, T)
        ctx.save_for_backward(ex, slot_o, off_o, cnt_o, ids, slot, off, cnt, row_src, idx, xp, h, act, y_src, ident,
                              weights, w13, w2)
        ctx.xch, ctx.block = xch, block
        return out

    @staticmethod
    def backward(ctx, dout):
        (ex, slot_o, off_o, cnt_o, ids, slot, off, cnt, row_src, idx, xp, h, act, y_src, ident, weights, w13,
         w2) = ctx.saved_tensors
        xch = ctx.xch
        T = dout.shape[0]
        dw = _bwd_dispatch(dout, y_src, ident, weights, ex, slot_o, off_o, cnt_o, w13.shape[0], xch)
        xch.barrier()
        g13, g2 = _bwd_owner(xch, ids, slot, off, row_src, idx, xp, h, act, w13, w2, ctx.block)
        xch.barrier()
        dx = _bwd_collect(xch, ident, T)
        gw13 = None if getattr(w13, "main_grad", None) is not None else g13.to(w13.dtype)
        gw2 = None if getattr(w2, "main_grad", None) is not None else g2.to(w2.dtype)
        return dx, dw, None, gw13, gw2, None, None


def ep_moe_forward(moe, x: torch.Tensor, weights: torch.Tensor, experts: torch.Tensor) -> torch.Tensor:
    """Routed-expert output for the local tokens ``x [T, D]`` under expert parallelism."""
    xch = getattr(moe, "ep_exchange", None)
    if xch is not None and x.is_cuda:
        return _PeerExperts.apply(x, weights, experts.to(torch.int32), moe.w13, moe.w2, xch, moe.args.swiglu_block)
    return _collective_forward(moe, x, weights, experts)


def _collective_forward(moe, x: torch.Tensor, weights: torch.Tensor, experts: torch.Tensor) -> torch.Tensor:
    """All-to-all transport (gloo on CPU, or EP groups that span nodes)."""
    from ..models.moe import moe_experts

    group = moe.ep_group
    ep = dist.get_world_size(group)
    E_local = moe.w13.shape[0]
    T, k = experts.shape
    flat_e = experts.reshape(-1).long()
    flat_w = weights.reshape(-1)
    tok = torch.arange(T, device=x.device).repeat_interleave(k)
    dest = flat_e // E_local
    order = torch.argsort(dest, stable=True)
    flat_e, flat_w, tok, dest = flat_e[order], flat_w[order], tok[order], dest[order]
    send = torch.bincount(dest, minlength=ep).to(torch.int64)
    recv = _exchange_splits(send, group)
    send_l = send.tolist()
    xs = all_to_all(x.index_select(0, tok), send_l, recv, group)
    es = all_to_all(flat_e.unsqueeze(-1), send_l, recv, group).squeeze(-1)
    # every received row goes through exactly one local expert with weight 1; the routing weight is
    # applied at the source after the combine
    ones = torch.ones(xs.shape[0], 1, dtype=torch.float32, device=x.device)
    ys = moe_experts(xs, ones, es.unsqueeze(-1), moe.w13, moe.w2, moe.args.swiglu_block,
                     expert_offset=moe.expert_offset)
    back = all_to_all(ys, recv, send_l, group)
    out = torch.zeros_like(x)
    return out.index_add(0, tok, back * flat_w.unsqueeze(-1).to(x.dtype))


def shard_experts(model, group, max_tokens: int | None = None) -> None:
    """Keep this EP rank's slice of every MoE layer's experts (call before flattening the parameters).

    On a CUDA model whose EP group fits one node, the layers also share one :class:`PeerExchange` sized
    for ``max_tokens`` tokens per layer call (collective: every rank calls this at set-up)."""
    import torch.nn as nn

    ep = dist.get_world_size(group)
    r = dist.get_rank(group)
    xch = None
    first = next((l.moe for l in model.layers if getattr(l, "moe", None) is not None), None)
    if first is not None and first.w13.is_cuda and max_tokens and dist.get_backend(group) == "nccl":
        from .symm import SymmetricHeap

        if SymmetricHeap.supported(group):
            xch = PeerExchange(group, first.w13.shape[2], int(max_tokens) * first.top_k, first.w13.device)
    for layer in model.layers:
        moe = getattr(layer, "moe", None)
        if moe is None:
            continue
        E = moe.w13.shape[0]
        if E % ep:
            raise ValueError(f"{E} experts do not divide over EP={ep}")
        n = E // ep
        with torch.no_grad():
            moe.w13 = nn.Parameter(moe.w13[r * n:(r + 1) * n].clone())
            moe.w2 = nn.Parameter(moe.w2[r * n:(r + 1) * n].clone())
        moe.expert_offset = r * n
        moe.ep_group = group
        moe.ep_exchange = xch


__all__ = ["PeerExchange", "all_to_all", "ep_moe_forward", "shard_experts"]
