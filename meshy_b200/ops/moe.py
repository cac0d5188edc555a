"""Mixture-of-experts layer on the native kernels, with no host synchronisation.

Forward of one layer on ``x [T, D]`` (k experts per token, E experts):

1. router logits ``x W_r^T`` (tcgen05 GEMM), then ``moe_route``: softmax over
   E, top-k, optional renormalisation -> ``weights [T, k]``, ``experts [T, k]``;
2. ``moe_plan``: per-expert counts, 128-row-aligned segment offsets ``off``
   (device tensor), the destination row of every (token, slot) assignment,
   and the gather of the token rows into the segments (zero padding rows);
3. two grouped GEMMs (``gemm_grouped`` mode GRP_M): gate/up with the SwiGLU
   epilogue, then down -- each 128-row tile reads the weights of the expert
   that owns it, located on the device from ``off``;
4. ``moe_combine``: ``out[t] = sum_j w[t, j] * y[row(t, j)]``.

Backward mirrors it: combine backward (expert-row gradients and routing-weight
gradients), grouped data-gradient GEMMs (B MN-major), grouped weight-gradient
GEMMs (mode GRP_K: contraction over each expert's segment, accumulated in fp32
straight into ``main_grad``), SwiGLU backward, gather-sum back to tokens, and
the router backward kernel.

The dispatched buffers are sized for the largest possible plan
(``T * k + E * 127`` rows, rounded to 128); the GEMMs skip the tiles past the
real end, which only the device knows. That keeps a decode step capturable in
a CUDA graph.

Reference semantics: torchtitan's MoE (``TT:torchtitan/models/common/moe.py``,
softmax router, top-k, optional ``route_norm``), which the reference trains.
"""

from __future__ import annotations

import torch

from ._ext import ext

GRP_M, GRP_K = 1, 2
EPI_STORE, EPI_SWIGLU = 0, 1


def plan_rows(n_assign: int, n_experts: int) -> int:
    """Rows of the dispatched buffers: every segment padded to 128 rows, at most ``E * 127`` padding."""
    return (n_assign + n_experts * 127 + 127) // 128 * 128


class _Route(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, k: int, norm: bool):
        C = ext()
        T, E = logits.shape
        probs = torch.empty(T, E, dtype=torch.float32, device=logits.device)
        weights = torch.empty(T, k, dtype=torch.float32, device=logits.device)
        experts = torch.empty(T, k, dtype=torch.int32, device=logits.device)
        C.moe_route(logits.contiguous(), k, norm, probs, weights, experts)
        ctx.save_for_backward(probs, weights, experts)
        ctx.norm = norm
        ctx.mark_non_differentiable(experts)
        return weights, experts

    @staticmethod
    def backward(ctx, dw, _de):
        probs, weights, experts = ctx.saved_tensors
        dlogits = torch.empty(probs.shape, dtype=torch.bfloat16, device=probs.device)
        if dw is None:
            dw = torch.zeros_like(weights)
        ext().moe_route_bwd(dw.float().contiguous(), probs, weights, experts, ctx.norm, dlogits)
        return dlogits, None, None


def route(logits: torch.Tensor, k: int, norm: bool):
    """``(weights [T, k] fp32, experts [T, k] int32)`` from bf16 router logits ``[T, E]``."""
    return _Route.apply(logits, k, norm)


def _wgrad_target(w: torch.Tensor):
    mg = getattr(w, "main_grad", None)
    if mg is not None:
        return mg, None
    buf = torch.zeros(w.shape, dtype=torch.float32, device=w.device)
    return buf, buf


class _Experts(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weights, experts, w13, w2, block: int):
        C = ext()
        T, D = x.shape
        k = experts.shape[1]
        E, F2, _ = w13.shape
        rows = plan_rows(T * k, E)
        dev = x.device
        cnt = torch.empty(E, dtype=torch.int32, device=dev)
        off = torch.empty(E + 1, dtype=torch.int32, device=dev)
        slot = torch.empty(T * k, dtype=torch.int32, device=dev)
        row_src = torch.empty(rows, dtype=torch.int32, device=dev)
        xp = torch.empty(rows, D, dtype=x.dtype, device=dev)
        C.moe_plan(experts.contiguous(), cnt, off, slot, row_src, x.contiguous(), xp)
        need_grad = ctx.needs_input_grad[0] or ctx.needs_input_grad[1] or ctx.needs_input_grad[3]
        h = torch.empty(rows, F2, dtype=x.dtype, device=dev) if need_grad else None
        act = torch.empty(rows, F2 // 2, dtype=x.dtype, device=dev)
        C.gemm_grouped(xp, w13, act, off, GRP_M, False, EPI_SWIGLU, h)
        y = torch.empty(rows, D, dtype=x.dtype, device=dev)
        C.gemm_grouped(act, w2, y, off, GRP_M, False, EPI_STORE, None)
        out = torch.empty(T, D, dtype=x.dtype, device=dev)
        C.moe_combine(y, slot, weights.contiguous(), out)
        if need_grad:
            ctx.save_for_backward(xp, h, act, y, slot, off, cnt, weights, w13, w2)
        ctx.block = block
        return out

    @staticmethod
    def backward(ctx, dout):
        C = ext()
        xp, h, act, y, slot, off, cnt, weights, w13, w2 = ctx.saved_tensors
        rows, D = y.shape
        T, k = weights.shape
        E, F2, _ = w13.shape
        dev = y.device
        dout = dout.contiguous()
        dy = torch.empty(rows, D, dtype=y.dtype, device=dev)
        dw = torch.empty(T, k, dtype=torch.float32, device=dev)
        C.moe_combine_bwd(dout, y, slot, weights, dy, dw)
        C.moe_zero_pad(off, cnt, dy)
        # down projection: d act = dy . W2_e ; dW2_e += dy_e^T act_e
        dact = torch.empty(rows, F2 // 2, dtype=y.dtype, device=dev)
        C.gemm_grouped(dy, w2, dact, off, GRP_M, True, EPI_STORE, None)
        g2, ret2 = _wgrad_target(w2)
        C.gemm_grouped(dy, act, g2.view(E * D, F2 // 2), off, GRP_K, True, EPI_STORE, None)
        # SwiGLU, gate/up projection: d xp = dh . W13_e ; dW13_e += dh_e^T xp_e
        dh = torch.empty_like(h)
        C.swiglu_bwd(h, dact, dh, ctx.block)
        dxp = torch.empty(rows, D, dtype=y.dtype, device=dev)
        C.gemm_grouped(dh, w13, dxp, off, GRP_M, True, EPI_STORE, None)
        g13, ret13 = _wgrad_target(w13)
        C.gemm_grouped(dh, xp, g13.view(E * F2, D), off, GRP_K, True, EPI_STORE, None)
        dx = torch.empty(T, D, dtype=y.dtype, device=dev)
        C.moe_combine(dxp, slot, None, dx)
        return (dx, dw, None, None if ret13 is None else ret13.to(w13.dtype),
                None if ret2 is None else ret2.to(w2.dtype), None)


def experts_forward(x, weights, experts, w13, w2, block: int):
    """Routed-expert output ``sum_j w[t, j] * SwiGLU_{e_tj}(x[t])`` on the native kernels."""
    from .checks import check_range

    check_range("MoE expert ids", experts, 0, w13.shape[0])
    return _Experts.apply(x, weights, experts, w13, w2, block)


__all__ = ["experts_forward", "plan_rows", "route"]
