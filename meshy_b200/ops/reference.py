"""Plain-PyTorch definitions of every hot op.

These are the numerical oracle for the CUDA kernels (tests compare each
kernel with the function of the same name here, computed in fp32) and the
implementation used when tensors live on the CPU (the CPU
``gloo`` tests).  They favour clarity over speed.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F


# ── normalisation ────────────────────────────────────────────────────────────

def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (y * w.float()).to(x.dtype)


# ── rotary embedding (rotate-half pairing) ───────────────────────────────────

def rope_cos_sin(positions: torch.Tensor, head_dim: int, theta: float) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin tables ``[T, head_dim/2]`` (fp32) for integer ``positions``."""
    # HF convention, fp32 throughout: inv_freq = 1 / theta^(arange(0, hd, 2) / hd)
    # built on the positions' device so the op can run inside CUDA graph capture
    dev = positions.device
    ar = torch.arange(0, head_dim, 2, dtype=torch.int64, device=dev).float() / head_dim
    inv = 1.0 / torch.pow(torch.full((), float(theta), device=dev), ar)
    ang = positions.float().unsqueeze(-1) * inv
    return torch.cos(ang), torch.sin(ang)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotate ``x [T, H, hd]``: pairs ``(i, i + hd/2)``."""
    half = x.shape[-1] // 2
    xf = x.float()
    x1, x2 = xf[..., :half], xf[..., half:]
    c = cos.unsqueeze(1)
    s = sin.unsqueeze(1)
    out = torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)
    return out.to(x.dtype)


# ── SwiGLU with the block-interleaved fused gate/up weight ───────────────────

def deinterleave_w13(h: torch.Tensor, block: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Split ``h [.., 2F]`` laid out ``[g0 u0 g1 u1 ...]`` (blocks of ``block``)."""
    shp = h.shape[:-1]
    two_f = h.shape[-1]
    hb = h.reshape(*shp, two_f // (2 * block), 2, block)
    g = hb[..., 0, :].reshape(*shp, two_f // 2)
    u = hb[..., 1, :].reshape(*shp, two_f // 2)
    return g, u


def interleave_w13(w_gate: torch.Tensor, w_up: torch.Tensor, block: int) -> torch.Tensor:
    """Inverse of :func:`deinterleave_w13` for weights ``[F, D]`` → ``[2F, D]``."""
    F_, D = w_gate.shape
    if F_ % block:
        raise ValueError(f"ffn dim {F_} is not a multiple of the interleave block {block}")
    g = w_gate.reshape(F_ // block, 1, block, D)
    u = w_up.reshape(F_ // block, 1, block, D)
    return torch.cat([g, u], dim=1).reshape(2 * F_, D)


def split_w13(w13: torch.Tensor, block: int) -> tuple[torch.Tensor, torch.Tensor]:
    two_f, D = w13.shape
    wb = w13.reshape(two_f // (2 * block), 2, block, D)
    return wb[:, 0].reshape(two_f // 2, D), wb[:, 1].reshape(two_f // 2, D)


def swiglu(h: torch.Tensor, block: int) -> torch.Tensor:
    g, u = deinterleave_w13(h.float(), block)
    return (F.silu(g) * u).to(h.dtype)


# ── attention ────────────────────────────────────────────────────────────────

def attention_chunks(q, k, v, cu_q, cu_k, q_off, scale: float | None = None) -> torch.Tensor:
    """Causal GQA attention of query chunks against separate key documents: chunk ``d`` holds queries
    ``cu_q[d]..`` at key positions ``q_off[d]..`` of keys ``cu_k[d]..cu_k[d+1]`` (fp32 oracle)."""
    T, Hq, hd = q.shape
    rep = Hq // k.shape[1]
    scale = scale if scale is not None else 1.0 / math.sqrt(hd)
    out = torch.zeros(T, Hq, hd, dtype=torch.float32, device=q.device)
    cq, ck, qo = cu_q.tolist(), cu_k.tolist(), q_off.tolist()
    for d in range(len(cq) - 1):
        s, e, ks, ke = cq[d], cq[d + 1], ck[d], ck[d + 1]
        if e <= s:
            continue
        qd = q[s:e].float().transpose(0, 1)
        kd = k[ks:ke].float().transpose(0, 1).repeat_interleave(rep, 0)
        vd = v[ks:ke].float().transpose(0, 1).repeat_interleave(rep, 0)
        sc = torch.matmul(qd, kd.transpose(1, 2)) * scale
        qpos = torch.arange(e - s, device=q.device).unsqueeze(1) + qo[d]
        kpos = torch.arange(ke - ks, device=q.device).unsqueeze(0)
        sc = sc.masked_fill(kpos > qpos, float("-inf"))
        out[s:e] = torch.matmul(torch.softmax(sc, -1), vd).transpose(0, 1)
    return out


def attention_varlen(
    q: torch.Tensor,          # [T, Hq, hd]
    k: torch.Tensor,          # [T, Hkv, hd]
    v: torch.Tensor,          # [T, Hkv, hd]
    cu_seqlens: torch.Tensor,  # [n_docs+1] int32
    scale: float | None = None,
    causal: bool = True,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Causal GQA attention over packed documents; returns ``(out, lse [Hq, T])``."""
    T, Hq, hd = q.shape
    Hkv = k.shape[1]
    rep = Hq // Hkv
    scale = scale if scale is not None else 1.0 / math.sqrt(hd)
    out = torch.zeros(T, Hq, hd, dtype=torch.float32, device=q.device)
    lse = torch.full((Hq, T), float("-inf"), dtype=torch.float32, device=q.device)
    cu = cu_seqlens.tolist()
    for i in range(len(cu) - 1):
        s, e = cu[i], cu[i + 1]
        if e <= s:
            continue
        qd = q[s:e].float().transpose(0, 1)                       # [Hq, L, hd]
        kd = k[s:e].float().transpose(0, 1).repeat_interleave(rep, 0)
        vd = v[s:e].float().transpose(0, 1).repeat_interleave(rep, 0)
        sc = torch.matmul(qd, kd.transpose(1, 2)) * scale          # [Hq, L, L]
        if causal:
            L = e - s
            m = torch.ones(L, L, dtype=torch.bool, device=q.device).triu(1)
            sc = sc.masked_fill(m, float("-inf"))
        l = torch.logsumexp(sc, dim=-1)                             # [Hq, L]
        p = torch.exp(sc - l.unsqueeze(-1))
        out[s:e] = torch.matmul(p, vd).transpose(0, 1)
        lse[:, s:e] = l
    return out.to(q.dtype), lse


def attention_decode_paged(
    q: torch.Tensor,            # [B, Hq, hd]
    k_cache: torch.Tensor,      # [n_pages, Hkv, page, hd]
    v_cache: torch.Tensor,
    block_table: torch.Tensor,  # [B, max_pages] int32
    seq_lens: torch.Tensor,     # [B] int32 (tokens in cache incl. current)
    scale: float | None = None,
) -> torch.Tensor:
    B, Hq, hd = q.shape
    Hkv, page = k_cache.shape[1], k_cache.shape[2]
    rep = Hq // Hkv
    scale = scale if scale is not None else 1.0 / math.sqrt(hd)
    out = torch.zeros(B, Hq, hd, dtype=torch.float32, device=q.device)
    for b in range(B):
        L = int(seq_lens[b])
        npg = (L + page - 1) // page
        pages = block_table[b, :npg].long()
        kk = k_cache[pages].permute(1, 0, 2, 3).reshape(Hkv, npg * page, hd)[:, :L].float()
        vv = v_cache[pages].permute(1, 0, 2, 3).reshape(Hkv, npg * page, hd)[:, :L].float()
        kk = kk.repeat_interleave(rep, 0)
        vv = vv.repeat_interleave(rep, 0)
        sc = torch.einsum("hd,hld->hl", q[b].float(), kk) * scale
        p = torch.softmax(sc, dim=-1)
        out[b] = torch.einsum("hl,hld->hd", p, vv)
    return out.to(q.dtype)


# ── LM head + log-softmax + entropy ──────────────────────────────────────────

def lm_head_logprobs(
    h: torch.Tensor,       # [T, D]
    w: torch.Tensor,       # [V, D]
    labels: torch.Tensor,  # [T] long
    with_entropy: bool = True,
    chunk: int = 1024,
) -> tuple[torch.Tensor, torch.Tensor | None]:
    """``lp[t] = z[t, y_t] - logsumexp(z[t])`` and entropy, chunked over tokens."""
    lps, ents = [], []
    for s in range(0, h.shape[0], chunk):
        z = (h[s:s + chunk].float() @ w.float().t())
        lse = torch.logsumexp(z, dim=-1)
        lps.append(z.gather(-1, labels[s:s + chunk].long().unsqueeze(-1)).squeeze(-1) - lse)
        if with_entropy:
            p = torch.softmax(z, dim=-1)
            ents.append(lse - (p * z).sum(-1))
    lp = torch.cat(lps) if lps else h.new_zeros(0, dtype=torch.float32)
    ent = (torch.cat(ents) if ents else h.new_zeros(0, dtype=torch.float32)) if with_entropy else None
    return lp, ent


# ── sampling ────────────────────────────────────────────────────────────────

def sample_with_logprob(logits: torch.Tensor, temperature: float, generator=None,
                        top_k: int = -1, top_p: float = 1.0) -> tuple[torch.Tensor, torch.Tensor]:
    """Multinomial sample from ``softmax(logits / T)`` (+ top-k / top-p filter).

    Returns the token and its log-probability under the *filtered, tempered*
    distribution, which is what the rollout reports as the behaviour policy.
    """
    z = logits.float()
    if temperature <= 0:
        tok = z.argmax(-1)
        return tok, torch.zeros_like(tok, dtype=torch.float32)
    z = z / temperature
    if top_k > 0:
        kth = torch.topk(z, top_k, dim=-1).values[..., -1:]
        z = z.masked_fill(z < kth, float("-inf"))
    if top_p < 1.0:
        sz, idx = torch.sort(z, dim=-1, descending=True)
        cp = torch.softmax(sz, -1).cumsum(-1)
        drop = (cp - torch.softmax(sz, -1)) > top_p
        sz = sz.masked_fill(drop, float("-inf"))
        z = torch.full_like(z, float("-inf")).scatter(-1, idx, sz)
    logp = torch.log_softmax(z, dim=-1)
    tok = torch.multinomial(logp.exp(), 1, generator=generator).squeeze(-1)
    return tok, logp.gather(-1, tok.unsqueeze(-1)).squeeze(-1)


# ── PPO clipped loss (token level) ──────────────────────────────────────────

def ppo_token_terms(new_lp, old_lp, adv_tok, mask, eps_low, eps_high):
    """Per-token ``-min(r A, clip(r) A) * mask`` and the ratio."""
    ratio = torch.exp(new_lp - old_lp)
    pg = -torch.minimum(ratio * adv_tok, ratio.clamp(1 - eps_low, 1 + eps_high) * adv_tok)
    return pg * mask, ratio


# ── optimiser ───────────────────────────────────────────────────────────────

def adamw_(param, grad, exp_avg, exp_avg_sq, *, lr, beta1, beta2, eps, weight_decay, step, grad_scale=1.0):
    """Decoupled-weight-decay Adam on fp32 tensors, in place."""
    g = grad * grad_scale
    exp_avg.mul_(beta1).add_(g, alpha=1 - beta1)
    exp_avg_sq.mul_(beta2).addcmul_(g, g, value=1 - beta2)
    bc1 = 1 - beta1 ** step
    bc2 = 1 - beta2 ** step
    param.mul_(1 - lr * weight_decay)
    denom = (exp_avg_sq / bc2).sqrt_().add_(eps)
    param.addcdiv_(exp_avg, denom, value=-lr / bc1)


__all__ = [n for n in dir() if not n.startswith("_") and n not in ("math", "torch", "F", "annotations")]
