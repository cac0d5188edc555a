"""Differentiable hot ops.

Each op has two bodies:

* CUDA tensors run the hand-written sm_100a kernels of ``meshy_b200._C``
  (tcgen05/TMEM GEMMs with fused epilogues, fused norm/rope kernels, flash
  attention, the fused LM-head log-prob kernel).  Weight gradients are
  accumulated in fp32 straight into ``param.main_grad`` by the wgrad GEMM
  epilogue (no bf16 weight-gradient tensor is ever formed).
* CPU tensors run :mod:`meshy_b200.ops.reference` under ordinary autograd.
  That is the fp32 oracle and the BASELINE config-1 CPU path.

A third body exists only for the comparison baseline: when
``set_torch_baseline(True)`` is active, CUDA tensors also take the PyTorch
path (cuBLAS GEMMs, torch SDPA).  The product never enables it.
"""

from __future__ import annotations

import math
from contextlib import contextmanager

import torch
import torch.nn.functional as F

from . import reference as ref
from ._ext import ext

_TORCH_BASELINE = False


def set_torch_baseline(flag: bool) -> None:
    global _TORCH_BASELINE
    _TORCH_BASELINE = bool(flag)


@contextmanager
def torch_baseline(flag: bool = True):
    old = _TORCH_BASELINE
    set_torch_baseline(flag)
    try:
        yield
    finally:
        set_torch_baseline(old)


def native(t: torch.Tensor) -> bool:
    """Whether ``t`` is handled by the native kernels."""
    return t.is_cuda and not _TORCH_BASELINE


def _acc_main_grad(w: torch.Tensor) -> torch.Tensor | None:
    return getattr(w, "main_grad", None)


# ═══════════════════════════════ linear ══════════════════════════════════════

EPI_NONE, EPI_SWIGLU = 0, 1


class _Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b, residual):
        C = ext()
        x2 = x.reshape(-1, x.shape[-1])
        out = torch.empty(x2.shape[0], w.shape[0], dtype=x.dtype, device=x.device)
        r2 = residual.reshape(-1, w.shape[0]) if residual is not None else None
        C.gemm(x2, w, out, False, False, b, r2, None, EPI_NONE, False, 0)
        ctx.save_for_backward(x2, w)
        ctx.has_b = b is not None
        ctx.bias_main_grad = _acc_main_grad(b) if b is not None else None
        ctx.has_r = residual is not None
        ctx.shape = x.shape
        return out.reshape(*x.shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, gy):
        C = ext()
        x2, w = ctx.saved_tensors
        gy2 = gy.reshape(-1, w.shape[0]).contiguous()
        gx = torch.empty_like(x2)
        # dX[T,K] = dY[T,N] · W[N,K]  (B operand is MN-major)
        C.gemm(gy2, w, gx, False, True, None, None, None, EPI_NONE, False, 0)
        gw = _wgrad(gy2, x2, w)
        gb = None
        if ctx.has_b:
            bsum = gy2.float().sum(0)
            mgb = getattr(ctx, "bias_main_grad", None)
            if mgb is not None:
                mgb.add_(bsum)
            else:
                gb = bsum.to(gy.dtype)
        gr = gy if ctx.has_r else None
        return gx.reshape(ctx.shape), gw, gb, gr


def _wgrad(gy2: torch.Tensor, x2: torch.Tensor, w: torch.Tensor):
    """``dW[N,K] += dY[T,N]^T X[T,K]`` (both operands MN-major)."""
    C = ext()
    mg = _acc_main_grad(w)
    if mg is not None:
        C.gemm(gy2, x2, mg, True, True, None, None, None, EPI_NONE, True, 0)
        return None
    gw = torch.zeros(w.shape, dtype=torch.float32, device=w.device)
    C.gemm(gy2, x2, gw, True, True, None, None, None, EPI_NONE, True, 0)
    return gw.to(w.dtype)


def linear(x, w, b=None, residual=None):
    """``y = x @ w.T (+ b) (+ residual)``."""
    if native(x):
        return _Linear.apply(x, w, b, residual)
    y = F.linear(x, w, b)
    return y + residual if residual is not None else y


class _LinearSwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w13, block):
        C = ext()
        x2 = x.reshape(-1, x.shape[-1])
        T = x2.shape[0]
        a = torch.empty(T, w13.shape[0] // 2, dtype=x.dtype, device=x.device)
        h = torch.empty(T, w13.shape[0], dtype=x.dtype, device=x.device)
        C.gemm(x2, w13, a, False, False, None, None, h, EPI_SWIGLU, False, block)
        ctx.save_for_backward(x2, w13, h)
        ctx.block = block
        ctx.shape = x.shape
        return a.reshape(*x.shape[:-1], a.shape[-1])

    @staticmethod
    def backward(ctx, ga):
        C = ext()
        x2, w13, h = ctx.saved_tensors
        ga2 = ga.reshape(h.shape[0], -1).contiguous()
        dh = torch.empty_like(h)
        C.swiglu_bwd(h, ga2, dh, ctx.block)
        gx = torch.empty_like(x2)
        C.gemm(dh, w13, gx, False, True, None, None, None, EPI_NONE, False, 0)
        gw = _wgrad(dh, x2, w13)
        return gx.reshape(ctx.shape), gw, None


def linear_swiglu(x, w13, block: int):
    """``silu(x Wg^T) * (x Wu^T)`` with the block-interleaved fused weight."""
    if native(x):
        if torch.is_grad_enabled() and (x.requires_grad or w13.requires_grad):
            return _LinearSwiGLU.apply(x, w13, block)
        # inference: the pre-activation is only needed by backward, so it is never written
        x2 = x.reshape(-1, x.shape[-1])
        a = torch.empty(x2.shape[0], w13.shape[0] // 2, dtype=x.dtype, device=x.device)
        ext().gemm(x2, w13, a, False, False, None, None, None, EPI_SWIGLU, False, block)
        return a.reshape(*x.shape[:-1], a.shape[-1])
    return ref.swiglu(F.linear(x, w13), block)


_FUSED_NORM = __import__("os").environ.get("MESHY_FUSED_NORM", "0") == "1"


def rmsnorm_linear(x, norm_w, eps, w, b=None, *, swiglu_block: int = 0):
    """Inference: ``linear(rmsnorm(x), w, b)`` (or the SwiGLU linear with ``swiglu_block``).

    With ``MESHY_FUSED_NORM=1`` the norm runs inside the small-M GEMM (each CTA recomputes the row
    rstd and rewrites its X tiles in shared memory).  Measured on B200 for the 1.5B model it is no
    faster at batch 8 and 33% slower at batch 64 than the separate RMSNorm kernel (the per-CTA rstd
    pass over the whole row block is on the critical path), so the two-kernel form is the default."""
    if _FUSED_NORM and native(x) and not torch.is_grad_enabled():
        x2 = x.reshape(-1, x.shape[-1])
        n_out = w.shape[0] // 2 if swiglu_block else w.shape[0]
        out = torch.empty(x2.shape[0], n_out, dtype=x.dtype, device=x.device)
        if ext().gemm_norm(x2, norm_w, float(eps), w, out, b, None, EPI_SWIGLU if swiglu_block else EPI_NONE,
                           int(swiglu_block)):
            return out.reshape(*x.shape[:-1], n_out)
    h = rmsnorm(x, norm_w, eps)
    if swiglu_block:
        return linear_swiglu(h, w, swiglu_block)
    return linear(h, w, b)


# ═══════════════════════════════ RMSNorm ═════════════════════════════════════

class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps):
        C = ext()
        x2 = x.reshape(-1, x.shape[-1]).contiguous()
        y = torch.empty_like(x2)
        rstd = torch.empty(x2.shape[0], dtype=torch.float32, device=x.device)
        C.rmsnorm_fwd(x2, w, y, rstd, eps)
        ctx.save_for_backward(x2, w, rstd)
        ctx.shape = x.shape
        return y.reshape(x.shape)

    @staticmethod
    def backward(ctx, gy):
        C = ext()
        x2, w, rstd = ctx.saved_tensors
        gx = torch.empty_like(x2)
        mg = _acc_main_grad(w)
        gw32 = mg if mg is not None else torch.zeros(w.shape, dtype=torch.float32, device=w.device)
        C.rmsnorm_bwd(gy.reshape(x2.shape).contiguous(), x2, w, rstd, gx, gw32)
        gw = None if mg is not None else gw32.to(w.dtype)
        return gx.reshape(ctx.shape), gw, None


def rmsnorm(x, w, eps: float):
    if native(x):
        return _RMSNorm.apply(x, w, eps)
    return ref.rmsnorm(x, w, eps)


# ═══════════════════════ QKV split + QK-norm + RoPE ══════════════════════════

class _QKVRope(torch.autograd.Function):
    """Split the fused QKV projection, apply QK-norm (optional) and RoPE.

    Output q ``[T, Hq, hd]``, k/v ``[T, Hkv, hd]`` (contiguous, ready for the
    attention kernel).
    """

    @staticmethod
    def forward(ctx, qkv, positions, qn, kn, n_heads, n_kv, hd, theta, eps):
        C = ext()
        T = qkv.shape[0]
        q = torch.empty(T, n_heads, hd, dtype=qkv.dtype, device=qkv.device)
        k = torch.empty(T, n_kv, hd, dtype=qkv.dtype, device=qkv.device)
        v = torch.empty(T, n_kv, hd, dtype=qkv.dtype, device=qkv.device)
        C.qkv_rope_fwd(qkv, positions, qn, kn, q, k, v, theta, eps)
        ctx.save_for_backward(qkv, positions, qn, kn)
        ctx.meta = (n_heads, n_kv, hd, theta, eps)
        return q, k, v

    @staticmethod
    def backward(ctx, gq, gk, gv):
        C = ext()
        qkv, positions, qn, kn = ctx.saved_tensors
        gqkv = torch.empty_like(qkv)
        n_heads, n_kv, hd, theta, eps = ctx.meta
        gqn = gkn = None
        if qn is not None:
            gqn = torch.zeros(qn.shape, dtype=torch.float32, device=qn.device)
            gkn = torch.zeros(kn.shape, dtype=torch.float32, device=kn.device)
        C.qkv_rope_bwd(qkv, positions, qn, kn, gq.contiguous(), gk.contiguous(), gv.contiguous(),
                       gqkv, gqn, gkn, theta, eps)
        if qn is not None:
            for w, g in ((qn, gqn), (kn, gkn)):
                mg = _acc_main_grad(w)
                if mg is not None:
                    mg.add_(g)
            gqn = None if _acc_main_grad(qn) is not None else gqn.to(qn.dtype)
            gkn = None if _acc_main_grad(kn) is not None else gkn.to(kn.dtype)
        return gqkv, None, gqn, gkn, None, None, None, None, None


def qkv_rope(qkv, positions, q_norm, k_norm, n_heads, n_kv, hd, theta, eps):
    if native(qkv):
        return _QKVRope.apply(qkv, positions, q_norm, k_norm, n_heads, n_kv, hd, theta, eps)
    T = qkv.shape[0]
    q = qkv[:, : n_heads * hd].reshape(T, n_heads, hd)
    k = qkv[:, n_heads * hd: (n_heads + n_kv) * hd].reshape(T, n_kv, hd)
    v = qkv[:, (n_heads + n_kv) * hd:].reshape(T, n_kv, hd)
    if q_norm is not None:
        q = ref.rmsnorm(q, q_norm, eps)
        k = ref.rmsnorm(k, k_norm, eps)
    cos, sin = ref.rope_cos_sin(positions, hd, theta)
    return ref.apply_rope(q, cos, sin), ref.apply_rope(k, cos, sin), v


# ═══════════════════════════════ attention ═══════════════════════════════════

class _FlashAttnVarlen(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, cu_seqlens, max_seqlen, scale):
        C = ext()
        out = torch.empty_like(q)
        lse = torch.empty(q.shape[1], q.shape[0], dtype=torch.float32, device=q.device)
        C.flash_attn_fwd(q, k, v, cu_seqlens, out, lse, int(max_seqlen), float(scale))
        ctx.save_for_backward(q, k, v, cu_seqlens, out, lse)
        ctx.meta = (int(max_seqlen), float(scale))
        return out

    @staticmethod
    def backward(ctx, gout):
        C = ext()
        q, k, v, cu, out, lse = ctx.saved_tensors
        max_seqlen, scale = ctx.meta
        gq = torch.empty_like(q)
        gk = torch.empty_like(k)
        gv = torch.empty_like(v)
        C.flash_attn_bwd(q, k, v, cu, out, gout.contiguous(), lse, gq, gk, gv, max_seqlen, scale)
        return gq, gk, gv, None, None, None


_ATTN_OVERRIDE: list = []


@contextmanager
def attention_override(fn):
    """Within the block, :func:`flash_attn_varlen` calls ``fn(q, k, v, cu_seqlens, max_seqlen, scale)``
    instead (context parallelism routes the model's attention through its sharder this way)."""
    _ATTN_OVERRIDE.append(fn)
    try:
        yield
    finally:
        _ATTN_OVERRIDE.pop()


def flash_attn_varlen(q, k, v, cu_seqlens, max_seqlen: int, scale: float | None = None):
    """Causal GQA attention over packed documents ``q [T,Hq,hd]``."""
    if _ATTN_OVERRIDE:
        return _ATTN_OVERRIDE[-1](q, k, v, cu_seqlens, max_seqlen, scale)
    scale = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    if native(q):
        return _FlashAttnVarlen.apply(q, k, v, cu_seqlens, max_seqlen, scale)
    if q.is_cuda and q.dtype != torch.float32:  # torch baseline: PyTorch's FlashAttention varlen kernel
        return _torch_varlen(q, k, v, cu_seqlens, max_seqlen, scale)
    return _RefAttn.apply(q, k, v, cu_seqlens, scale)  # CPU, and fp32 oracles on the GPU


def _torch_varlen(q, k, v, cu, max_seqlen, scale):
    """Comparison baseline: causal varlen attention through ``torch.nn.attention.varlen`` (FlashAttention
    inside PyTorch, differentiable, GQA by head count), else SDPA per document."""
    try:
        from torch.nn.attention.varlen import varlen_attn
    except ImportError:  # older PyTorch
        return _sdpa_varlen(q, k, v, cu, scale)
    cu32 = cu.to(torch.int32)
    return varlen_attn(q, k, v, cu32, cu32, int(max_seqlen), int(max_seqlen), scale=scale, window_size=(-1, 0))


class _FlashAttnKV(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, cu_q, cu_k, q_off, max_q, max_k, scale):
        C = ext()
        out = torch.empty_like(q)
        lse = torch.empty(q.shape[1], q.shape[0], dtype=torch.float32, device=q.device)
        C.flash_attn_fwd_kv(q, k, v, cu_q, cu_k, q_off, out, lse, int(max_q), float(scale))
        ctx.save_for_backward(q, k, v, cu_q, cu_k, q_off, out, lse)
        ctx.meta = (int(max_q), int(max_k), float(scale))
        return out

    @staticmethod
    def backward(ctx, gout):
        C = ext()
        q, k, v, cu_q, cu_k, q_off, out, lse = ctx.saved_tensors
        max_q, max_k, scale = ctx.meta
        gq, gk, gv = torch.empty_like(q), torch.zeros_like(k), torch.zeros_like(v)
        C.flash_attn_bwd_kv(q, k, v, cu_q, cu_k, q_off, out, gout.contiguous(), lse, gq, gk, gv, max_q, max_k, scale)
        return gq, gk, gv, None, None, None, None, None, None


def flash_attn_chunks(q, k, v, cu_q, cu_k, q_off, max_q: int, max_k: int, scale: float | None = None):
    """Causal attention of query chunks ``q [Tq, Hq, hd]`` against key documents ``k/v [Tk, Hkv, hd]``:
    chunk ``d`` = rows ``cu_q[d]..cu_q[d+1]`` sitting at key positions ``q_off[d]..`` of document
    ``cu_k[d]..cu_k[d+1]``.  Context parallelism runs its local head/tail chunks against the gathered
    sequence with it."""
    scale = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    if native(q):
        return _FlashAttnKV.apply(q, k, v, cu_q, cu_k, q_off, max_q, max_k, scale)
    return ref.attention_chunks(q, k, v, cu_q, cu_k, q_off, scale).to(q.dtype)


class _RefAttn(torch.autograd.Function):
    """CPU oracle wrapped so autograd sees one node (memory-light backward)."""

    @staticmethod
    def forward(ctx, q, k, v, cu, scale):
        ctx.save_for_backward(q, k, v, cu)
        ctx.scale = scale
        return ref.attention_varlen(q, k, v, cu, scale)[0]

    @staticmethod
    def backward(ctx, g):
        q, k, v, cu = ctx.saved_tensors
        with torch.enable_grad():
            qq, kk, vv = (t.detach().requires_grad_(True) for t in (q, k, v))
            o = ref.attention_varlen(qq, kk, vv, cu, ctx.scale)[0]
            gq, gk, gv = torch.autograd.grad(o, (qq, kk, vv), g)
        return gq, gk, gv, None, None


def _sdpa_varlen(q, k, v, cu, scale):
    outs = []
    rep = q.shape[1] // k.shape[1]
    for s, e in zip(cu[:-1].tolist(), cu[1:].tolist()):
        if e <= s:
            continue
        qd = q[s:e].transpose(0, 1).unsqueeze(0)
        kd = k[s:e].transpose(0, 1).repeat_interleave(rep, 0).unsqueeze(0)
        vd = v[s:e].transpose(0, 1).repeat_interleave(rep, 0).unsqueeze(0)
        o = F.scaled_dot_product_attention(qd, kd, vd, is_causal=True, scale=scale)
        outs.append(o.squeeze(0).transpose(0, 1))
    return torch.cat(outs, 0)


# ══════════════════════ LM head + log-prob + entropy ═════════════════════════

class _LMHeadLogprob(torch.autograd.Function):
    """Fused ``log softmax(h W^T)[y]`` (+ detached entropy) without [T,V] logits.

    Forward: one tcgen05 GEMM sweep over vocab tiles whose epilogue keeps the
    online (max, sum-exp, sum p·z, target logit) per row.  Backward recomputes
    the logits per token chunk, forms ``dz = g (onehot - softmax)`` in the GEMM
    epilogue, and feeds it to the dgrad/wgrad GEMMs.
    """

    @staticmethod
    def forward(ctx, h, w, labels, with_entropy, chunk):
        C = ext()
        T = h.shape[0]
        lp = torch.empty(T, dtype=torch.float32, device=h.device)
        lse = torch.empty(T, dtype=torch.float32, device=h.device)
        ent = torch.empty(T, dtype=torch.float32, device=h.device) if with_entropy else None
        C.lmhead_logprob_fwd(h, w, labels, lp, lse, ent)
        ctx.save_for_backward(h, w, labels, lse)
        ctx.chunk = chunk
        return lp, ent

    @staticmethod
    def backward(ctx, glp, gent):
        C = ext()
        h, w, labels, lse = ctx.saved_tensors
        T, D = h.shape
        V = w.shape[0]
        gh = torch.empty_like(h)
        mg = _acc_main_grad(w)
        gw32 = mg if mg is not None else torch.zeros(w.shape, dtype=torch.float32, device=w.device)
        glp = glp.contiguous().float()
        chunk = max(128, min(ctx.chunk, T))
        dz = torch.empty(min(chunk, T), V, dtype=h.dtype, device=h.device)
        for s in range(0, T, chunk):
            e = min(T, s + chunk)
            dzc = dz[: e - s]
            C.lmhead_dlogits(h[s:e], w, labels[s:e], lse[s:e], glp[s:e], dzc)
            C.gemm(dzc, w, gh[s:e], False, True, None, None, None, EPI_NONE, False, 0)
            C.gemm(dzc, h[s:e], gw32, True, True, None, None, None, EPI_NONE, True, 0)
        gw = None if mg is not None else gw32.to(w.dtype)
        return gh, gw, None, None, None


def lm_head_logprobs(h, w, labels, with_entropy: bool = True, chunk: int = 4096):
    from .checks import check_range

    check_range("LM-head labels", labels, 0, w.shape[0])
    if native(h):
        return _LMHeadLogprob.apply(h, w, labels, with_entropy, chunk)
    if h.is_cuda:  # torch baseline
        return _torch_lmhead_chunked(h, w, labels, with_entropy, chunk)
    return ref.lm_head_logprobs(h, w, labels, with_entropy, chunk=min(chunk, 1024))


def _torch_lmhead_chunked(h, w, labels, with_entropy, chunk):
    from torch.utils.checkpoint import checkpoint

    def lp_chunk(hc, yc):
        z = F.linear(hc, w).float()
        return -F.cross_entropy(z, yc, reduction="none")

    lps, ents = [], []
    for s in range(0, h.shape[0], chunk):
        hc, yc = h[s:s + chunk], labels[s:s + chunk]
        lps.append(checkpoint(lp_chunk, hc, yc, use_reentrant=False) if torch.is_grad_enabled() else lp_chunk(hc, yc))
        if with_entropy:
            with torch.no_grad():
                z = F.linear(hc, w).float()
                lse = torch.logsumexp(z, -1)
                ents.append(lse - (torch.softmax(z, -1) * z).sum(-1))
    return torch.cat(lps), (torch.cat(ents) if with_entropy else None)


# ═══════════════════════════════ embedding ═══════════════════════════════════

class _Embedding(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, w):
        C = ext()
        out = torch.empty(ids.shape[0], w.shape[1], dtype=w.dtype, device=w.device)
        C.embedding_fwd(ids, w, out)
        ctx.save_for_backward(ids)
        ctx.w = w
        return out

    @staticmethod
    def backward(ctx, g):
        C = ext()
        (ids,) = ctx.saved_tensors
        w = ctx.w
        mg = _acc_main_grad(w)
        gw32 = mg if mg is not None else torch.zeros(w.shape, dtype=torch.float32, device=w.device)
        C.embedding_bwd(ids, g.contiguous(), gw32)
        return None, (None if mg is not None else gw32.to(w.dtype))


def embedding(ids, w):
    from .checks import check_range

    check_range("embedding token ids", ids, 0, w.shape[0])
    if native(w):
        return _Embedding.apply(ids, w)
    return F.embedding(ids, w)


__all__ = [
    "embedding", "flash_attn_varlen", "linear", "linear_swiglu", "lm_head_logprobs", "native",
    "qkv_rope", "rmsnorm", "set_torch_baseline", "torch_baseline",
]
