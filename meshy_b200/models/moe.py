"""Mixture-of-experts feed-forward (Qwen3-MoE style).

Router: ``softmax(x W_r^T)`` over all experts, top-k, optional renormalisation
of the selected weights (``route_norm``), as in torchtitan's qwen3 MoE that
the reference trains (``TT:torchtitan/models/common/moe.py``).  Experts are
SwiGLU MLPs stored stacked: ``w13 [E, 2F, D]`` (block-interleaved gate/up, the
same layout as the dense block) and ``w2 [E, D, F]``.

On CUDA the router (softmax + top-k kernel), the device-side expert plan and
token gather, the grouped tcgen05 expert GEMMs and the weighted combine run
in the native kernels (:mod:`meshy_b200.ops.moe`), with no host
synchronisation. Under expert parallelism the tokens travel to the experts'
owners as described in :mod:`meshy_b200.parallel.ep`. On CPU the per-expert
loop of :func:`moe_experts` is the oracle.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from ..ops import functional as Fx
from ..ops import reference as ref
from .args import ModelArgs


def route(x: torch.Tensor, w_router: torch.Tensor, top_k: int, route_norm: bool):
    """Top-k routing: returns ``(weights [T,k] fp32, experts [T,k] int64)``."""
    scores = torch.softmax(Fx.linear(x, w_router).float(), dim=-1)
    w, e = torch.topk(scores, top_k, dim=-1)
    if route_norm:
        w = w / w.sum(-1, keepdim=True).clamp(min=1e-20)
    return w, e


class MoE(nn.Module):
    def __init__(self, args: ModelArgs):
        super().__init__()
        m = args.moe
        self.args = args
        self.n_experts = m.n_experts
        self.top_k = m.top_k
        self.route_norm = m.route_norm
        d, f = args.dim, m.expert_ffn_dim
        self.router = nn.Parameter(torch.empty(m.n_experts, d))
        self.w13 = nn.Parameter(torch.empty(m.n_experts, 2 * f, d))
        self.w2 = nn.Parameter(torch.empty(m.n_experts, d, f))
        if m.n_shared_experts:
            self.shared_w13 = nn.Parameter(torch.empty(2 * f * m.n_shared_experts, d))
            self.shared_w2 = nn.Parameter(torch.empty(d, f * m.n_shared_experts))
        else:
            self.shared_w13 = self.shared_w2 = None
        #: local expert range under expert parallelism (set by parallel.ep)
        self.expert_offset = 0
        self.ep_group = None
        #: inference expert parallelism over ranks that hold the same tokens (a tensor-parallel replica): each
        #: rank runs the assignments of its own experts and the outputs are summed over this group
        self.ep_tokens_group = None

    def reset_parameters(self, std: float, depth_std: float) -> None:
        nn.init.normal_(self.router, std=std)
        nn.init.normal_(self.w13, std=std)
        nn.init.normal_(self.w2, std=depth_std)
        if self.shared_w13 is not None:
            nn.init.normal_(self.shared_w13, std=std)
            nn.init.normal_(self.shared_w2, std=depth_std)

    def _replicated_token_experts(self, x, weights, experts):
        """Expert parallelism when every rank holds every token: assignments to other ranks' experts get weight 0
        (and a local expert id, so the device plan needs no host synchronisation), then the outputs of the ranks
        are summed."""
        import torch.distributed as dist

        e_local = self.w13.shape[0]
        local = experts.long() - self.expert_offset
        mine = (local >= 0) & (local < e_local)
        w = torch.where(mine, weights, torch.zeros_like(weights))
        e = torch.where(mine, local, torch.zeros_like(local)).to(experts.dtype)
        if Fx.native(x):
            from ..ops import moe as M

            out = M.experts_forward(x, w, e, self.w13, self.w2, self.args.swiglu_block)
        else:
            out = moe_experts(x, w, e, self.w13, self.w2, self.args.swiglu_block)
        out = out.float()
        dist.all_reduce(out, group=self.ep_tokens_group)
        return out.to(x.dtype)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.ep_tokens_group is not None:
            if Fx.native(x):
                from ..ops import moe as M

                weights, experts = M.route(Fx.linear(x, self.router), self.top_k, self.route_norm)
            else:
                weights, experts = route(x, self.router, self.top_k, self.route_norm)
            out = self._replicated_token_experts(x, weights, experts)
            if self.shared_w13 is not None:
                out = out + Fx.linear(Fx.linear_swiglu(x, self.shared_w13, self.args.swiglu_block), self.shared_w2)
            return out
        if Fx.native(x):
            from ..ops import moe as M

            weights, experts = M.route(Fx.linear(x, self.router), self.top_k, self.route_norm)
            if self.ep_group is not None:
                from ..parallel.ep import ep_moe_forward

                out = ep_moe_forward(self, x, weights, experts)
            else:
                out = M.experts_forward(x, weights, experts, self.w13, self.w2, self.args.swiglu_block)
            if self.shared_w13 is not None:
                out = out + Fx.linear(Fx.linear_swiglu(x, self.shared_w13, self.args.swiglu_block), self.shared_w2)
            return out
        weights, experts = route(x, self.router, self.top_k, self.route_norm)
        if self.ep_group is not None:
            from ..parallel.ep import ep_moe_forward

            out = ep_moe_forward(self, x, weights, experts)
        else:
            out = moe_experts(x, weights, experts, self.w13, self.w2, self.args.swiglu_block)
        if self.shared_w13 is not None:
            out = out + Fx.linear(Fx.linear_swiglu(x, self.shared_w13, self.args.swiglu_block), self.shared_w2)
        return out


def moe_experts(x, weights, experts, w13, w2, block: int, expert_offset: int = 0):
    """Sum over selected experts of ``weight * SwiGLU_e(x)`` (local experts only).

    Tokens are sorted by expert so each expert runs one GEMM over a contiguous
    slice (the grouped-GEMM formulation); tokens routed to experts outside
    ``[expert_offset, expert_offset + E_local)`` are skipped.
    """
    T, D = x.shape
    E_local = w13.shape[0]
    flat_e = experts.reshape(-1) - expert_offset
    flat_w = weights.reshape(-1)
    tok = torch.arange(T, device=x.device).repeat_interleave(experts.shape[1])
    keep = (flat_e >= 0) & (flat_e < E_local)
    flat_e, flat_w, tok = flat_e[keep], flat_w[keep], tok[keep]
    order = torch.argsort(flat_e, stable=True)
    flat_e, flat_w, tok = flat_e[order], flat_w[order], tok[order]
    counts = torch.bincount(flat_e, minlength=E_local).tolist()
    xs = x[tok]
    outs = []
    off = 0
    for e, c in enumerate(counts):
        if c == 0:
            continue
        xe = xs[off:off + c]
        w13e, w2e = w13[e], w2[e]
        if hasattr(w13, "main_grad"):  # route expert weight-grads into the flat fp32 buffer
            w13e.main_grad = w13.main_grad[e]
            w2e.main_grad = w2.main_grad[e]
        a = Fx.linear_swiglu(xe, w13e, block)
        outs.append(Fx.linear(a, w2e))
        off += c
    if not outs:
        return torch.zeros_like(x)
    y = torch.cat(outs, 0) * flat_w.unsqueeze(-1).to(x.dtype)
    out = torch.zeros_like(x)
    return out.index_add(0, tok, y)


__all__ = ["MoE", "moe_experts", "route"]
