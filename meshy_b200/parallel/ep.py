"""Expert parallelism: experts sharded over an EP group, tokens dispatched to their owners.

Expert ``e`` lives on EP rank ``e // E_local`` (``E_local = n_experts / ep``),
the layout torchtitan's ``ExpertParallel`` uses (experts sharded on dim 0,
``TT:torchtitan/distributed/expert_parallel.py:50-75``).  One MoE layer:

1. route (top-k of the softmax router) on the local tokens;
2. **dispatch**: every (token, expert) assignment is sent to the expert's
   owner with one ``all_to_all_single`` of the token rows (sorted by
   destination rank, split sizes exchanged first);
3. the owner runs its local experts over what it received (tokens grouped by
   expert, one expert GEMM pair each);
4. **combine**: outputs go back with the inverse ``all_to_all_single`` and are
   summed at the source with the routing weights.

Both all-to-alls are differentiable (autograd runs the inverse exchange in
backward).  They go through NCCL (gloo on CPU); fusing the dispatch into the
grouped GEMM over NVLink peer memory is the planned replacement.
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


def ep_moe_forward(moe, x: torch.Tensor, weights: torch.Tensor, experts: torch.Tensor) -> torch.Tensor:
    """Routed-expert output for the local tokens ``x [T, D]`` under expert parallelism."""
    from ..models.moe import moe_experts

    group = moe.ep_group
    ep = dist.get_world_size(group)
    E_local = moe.w13.shape[0]
    T, k = experts.shape
    flat_e = experts.reshape(-1)
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


def shard_experts(model, group) -> None:
    """Keep this EP rank's slice of every MoE layer's experts (call before flattening the parameters)."""
    import torch.nn as nn

    ep = dist.get_world_size(group)
    r = dist.get_rank(group)
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


__all__ = ["all_to_all", "ep_moe_forward", "shard_experts"]
