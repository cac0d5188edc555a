"""Numerics of every sm_100a kernel against the fp32 PyTorch definition of the same op."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

from meshy_b200.ops import reference as ref  # noqa: E402


def C():
    from meshy_b200.ops._ext import ext

    return ext()


def rel_err(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


DEV = "cuda"


def bf(*shape, scale=1.0):
    return (torch.randn(*shape, device=DEV) * scale).to(torch.bfloat16)


@pytest.mark.parametrize("M,N,K", [(256, 512, 384), (200, 384, 136), (1000, 1536, 1536), (3, 2048, 1536),
                                   (64, 1536, 8960), (4096, 2304, 1024)])
def test_gemm_tn(M, N, K):
    torch.manual_seed(0)
    a, b = bf(M, K), bf(N, K)
    out = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    C().gemm(a, b, out, False, False, None, None, None, 0, False, 0)
    torch.cuda.synchronize()
    assert C().device_error() == 0
    assert rel_err(out, a.float() @ b.float().t()) < 1e-2


@pytest.mark.parametrize("M,N,K", [(256, 512, 384), (130, 200, 72), (2048, 1536, 2048)])
def test_gemm_bias_residual_f32(M, N, K):
    torch.manual_seed(1)
    a, b, bias, res = bf(M, K), bf(N, K), bf(N), bf(M, N)
    out = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    C().gemm(a, b, out, False, False, bias, res, None, 0, False, 0)
    ref_ = a.float() @ b.float().t() + bias.float() + res.float()
    assert rel_err(out, ref_) < 1e-2
    out32 = torch.empty(M, N, dtype=torch.float32, device=DEV)
    C().gemm(a, b, out32, False, False, None, None, None, 0, False, 0)
    assert rel_err(out32, a.float() @ b.float().t()) < 5e-3


@pytest.mark.parametrize("T,N,K", [(512, 256, 384), (300, 1536, 1536), (4096, 1024, 2048), (4096, 2048, 1536)])
def test_gemm_dgrad_wgrad(T, N, K):
    torch.manual_seed(2)
    gy, w, x = bf(T, N), bf(N, K), bf(T, K)
    gx = torch.empty(T, K, dtype=torch.bfloat16, device=DEV)
    C().gemm(gy, w, gx, False, True, None, None, None, 0, False, 0)  # dX = dY W
    assert rel_err(gx, gy.float() @ w.float()) < 1e-2
    gw = torch.ones(N, K, dtype=torch.float32, device=DEV)
    C().gemm(gy, x, gw, True, True, None, None, None, 0, True, 0)  # dW += dY^T X
    assert rel_err(gw, 1.0 + gy.float().t() @ x.float()) < 5e-3
    # A MN-major, B K-major: out[N, K2] = gy^T [N, T] · y[K2, T]^T with y = x^T stored [K2, T]
    y = x.t().contiguous()
    out = torch.empty(N, K, dtype=torch.float32, device=DEV)
    if (T * 2) % 16 != 0:
        # a [K2, T] bf16 row of 600 bytes is not a legal TMA stride: the op must refuse, not misread
        with pytest.raises(RuntimeError, match="multiple of 16 bytes"):
            C().gemm(gy, y, out, True, False, None, None, None, 0, False, 0)
        return
    C().gemm(gy, y, out, True, False, None, None, None, 0, False, 0)
    assert rel_err(out, gy.float().t() @ x.float()) < 5e-3


def test_gemm_swiglu():
    torch.manual_seed(3)
    T, D, F = 700, 512, 768
    x, w13 = bf(T, D), bf(2 * F, D, scale=0.05)
    a = torch.empty(T, F, dtype=torch.bfloat16, device=DEV)
    h = torch.empty(T, 2 * F, dtype=torch.bfloat16, device=DEV)
    C().gemm(x, w13, a, False, False, None, None, h, 1, False, 64)
    h_ref = x.float() @ w13.float().t()
    assert rel_err(h, h_ref) < 1e-2
    assert rel_err(a, ref.swiglu(h_ref, 64)) < 2e-2


def test_rmsnorm_fwd_bwd():
    torch.manual_seed(4)
    for D in (256, 1536, 4096):
        x = bf(333, D)
        w = (torch.rand(D, device=DEV) + 0.5).to(torch.bfloat16)
        y = torch.empty_like(x)
        rstd = torch.empty(333, device=DEV)
        C().rmsnorm_fwd(x, w, y, rstd, 1e-6)
        assert rel_err(y, ref.rmsnorm(x.float(), w.float(), 1e-6)) < 1e-2
        xr = x.float().requires_grad_(True)
        wr = w.float().requires_grad_(True)
        gy = bf(333, D)
        ref.rmsnorm(xr, wr, 1e-6).backward(gy.float())
        gx = torch.empty_like(x)
        gw = torch.zeros(D, device=DEV)
        C().rmsnorm_bwd(gy, x, w, rstd, gx, gw)
        assert rel_err(gx, xr.grad) < 2e-2
        assert rel_err(gw, wr.grad) < 2e-2


@pytest.mark.parametrize("qk_norm", [False, True])
def test_qkv_rope(qk_norm):
    torch.manual_seed(5)
    T, Hq, Hkv, hd = 77, 12, 2, 128
    qkv = bf(T, (Hq + 2 * Hkv) * hd)
    pos = torch.randint(0, 5000, (T,), device=DEV, dtype=torch.int32)
    qn = (torch.rand(hd, device=DEV) + 0.5).to(torch.bfloat16) if qk_norm else None
    kn = (torch.rand(hd, device=DEV) + 0.5).to(torch.bfloat16) if qk_norm else None
    from meshy_b200.ops import functional as Fx

    q, k, v = Fx.qkv_rope(qkv, pos, qn, kn, Hq, Hkv, hd, 1e6, 1e-6)
    with Fx.torch_baseline():
        qr, kr, vr = Fx.qkv_rope(qkv.float(), pos, None if qn is None else qn.float(),
                                 None if kn is None else kn.float(), Hq, Hkv, hd, 1e6, 1e-6)
    assert rel_err(q, qr) < 1e-2 and rel_err(k, kr) < 1e-2 and rel_err(v, vr) < 1e-3
    # backward
    qkv_r = qkv.float().requires_grad_(True)
    qn_r = qn.float().requires_grad_(True) if qk_norm else None
    kn_r = kn.float().requires_grad_(True) if qk_norm else None
    with Fx.torch_baseline():
        a, b, c = Fx.qkv_rope(qkv_r, pos, qn_r, kn_r, Hq, Hkv, hd, 1e6, 1e-6)
    gq, gk, gv = bf(T, Hq, hd), bf(T, Hkv, hd), bf(T, Hkv, hd)
    torch.autograd.backward([a, b, c], [gq.float(), gk.float(), gv.float()])
    gqkv = torch.empty_like(qkv)
    gqn = torch.zeros(hd, device=DEV) if qk_norm else None
    gkn = torch.zeros(hd, device=DEV) if qk_norm else None
    C().qkv_rope_bwd(qkv, pos, qn, kn, gq, gk, gv, gqkv, gqn, gkn, 1e6, 1e-6)
    assert rel_err(gqkv, qkv_r.grad) < 2e-2
    if qk_norm:
        assert rel_err(gqn, qn_r.grad) < 2e-2 and rel_err(gkn, kn_r.grad) < 2e-2


@pytest.mark.parametrize("hd,Hq,Hkv", [(128, 12, 2), (64, 4, 2)])
def test_flash_attn_fwd_bwd(hd, Hq, Hkv):
    torch.manual_seed(6)
    lens = [1, 63, 64, 65, 200, 37]
    T = sum(lens)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32, device=DEV)
    q, k, v = bf(T, Hq, hd), bf(T, Hkv, hd), bf(T, Hkv, hd)
    scale = 1 / math.sqrt(hd)
    out = torch.empty_like(q)
    lse = torch.empty(Hq, T, device=DEV)
    C().flash_attn_fwd(q, k, v, cu, out, lse, max(lens), scale)
    o_ref, lse_ref = ref.attention_varlen(q.float(), k.float(), v.float(), cu, scale)
    assert rel_err(out, o_ref) < 1e-2
    assert torch.allclose(lse, lse_ref, atol=1e-2, rtol=1e-3)
    # backward
    qr, kr, vr = (t.float().requires_grad_(True) for t in (q, k, v))
    o2, _ = ref.attention_varlen(qr, kr, vr, cu, scale)
    go = bf(T, Hq, hd)
    o2.backward(go.float())
    gq, gk, gv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    C().flash_attn_bwd(q, k, v, cu, out, go, lse, gq, gk, gv, max(lens), scale)
    assert rel_err(gq, qr.grad) < 3e-2
    assert rel_err(gk, kr.grad) < 3e-2
    assert rel_err(gv, vr.grad) < 3e-2


def test_paged_decode_and_kv_write():
    torch.manual_seed(7)
    B, Hq, Hkv, hd, page = 5, 12, 2, 128, 64
    n_pages = 64
    kc = torch.zeros(n_pages, Hkv, page, hd, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    lens = [1, 64, 65, 300, 1000]
    bt = torch.zeros(B, 20, dtype=torch.int32, device=DEV)
    perm = torch.randperm(n_pages - 1, device=DEV) + 1
    used = 0
    for b, L in enumerate(lens):
        npg = (L + page - 1) // page
        bt[b, :npg] = perm[used:used + npg].int()
        used += npg
        # write L tokens through kv_write
        k_new, v_new = bf(L, Hkv, hd), bf(L, Hkv, hd)
        slots = (bt[b, torch.arange(L, device=DEV) // page].long() * page + torch.arange(L, device=DEV) % page)
        C().kv_write(k_new, v_new, kc, vc, slots)
    seq = torch.tensor(lens, dtype=torch.int32, device=DEV)
    q = bf(B, Hq, hd)
    out = torch.empty_like(q)
    C().paged_attention(q, kc, vc, bt, seq, out, 1 / math.sqrt(hd), None)
    o_ref = ref.attention_decode_paged(q.float(), kc.float(), vc.float(), bt, seq, 1 / math.sqrt(hd))
    assert rel_err(out, o_ref) < 1e-2
    # decode-step mode (older pages loaded before the dependency wait): same result
    out2 = torch.empty_like(q)
    C().paged_attention(q, kc, vc, bt, seq, out2, 1 / math.sqrt(hd), None, True)
    torch.cuda.synchronize()
    assert C().device_error() == 0
    assert torch.equal(out2, out)


def test_lmhead_logprob_fwd_bwd():
    torch.manual_seed(8)
    T, D, V = 300, 256, 5000
    h, w = bf(T, D), bf(V, D, scale=0.2)
    labels = torch.randint(0, V, (T,), device=DEV)
    lp = torch.empty(T, device=DEV)
    lse = torch.empty(T, device=DEV)
    ent = torch.empty(T, device=DEV)
    C().lmhead_logprob_fwd(h, w, labels, lp, lse, ent)
    lp_ref, ent_ref = ref.lm_head_logprobs(h.float(), w.float(), labels, True)
    assert torch.allclose(lp, lp_ref, atol=2e-2, rtol=1e-3)
    assert torch.allclose(ent, ent_ref, atol=2e-2, rtol=1e-3)
    # backward through the op
    from meshy_b200.ops import functional as Fx

    hr = h.clone().requires_grad_(True)
    wr = w.clone().requires_grad_(True)
    lp2, _ = Fx.lm_head_logprobs(hr, wr, labels, False, chunk=128)
    g = torch.randn(T, device=DEV)
    lp2.backward(g)
    hf = h.float().requires_grad_(True)
    wf = w.float().requires_grad_(True)
    lpf, _ = ref.lm_head_logprobs(hf, wf, labels, False)
    lpf.backward(g)
    assert rel_err(hr.grad, hf.grad) < 3e-2
    assert rel_err(wr.grad, wf.grad) < 3e-2


def test_lmhead_sample_distribution():
    torch.manual_seed(9)
    B, D, V = 4, 64, 300
    h, w = bf(B, D), bf(V, D, scale=0.3)
    z = (h.float() @ w.float().t())
    p = torch.softmax(z, -1)
    counts = torch.zeros(B, V, device=DEV)
    step = torch.zeros(1, dtype=torch.int64, device=DEV)
    tok = torch.empty(B, dtype=torch.int64, device=DEV)
    lp = torch.empty(B, device=DEV)
    n = 4000
    for _ in range(n):
        C().lmhead_sample(h, w, tok, lp, 1.0, 1234, step)
        step += 1
        counts[torch.arange(B, device=DEV), tok] += 1
    assert torch.allclose(lp, torch.log(p.gather(1, tok[:, None]).squeeze(1)), atol=2e-2)
    emp = counts / n
    # total-variation distance of the empirical distribution
    tv = 0.5 * (emp - p).abs().sum(-1)
    assert (tv < 0.08).all(), tv


def test_lmhead_sample_small_distribution():
    """The small-M sampler (LM head on the swapped-operand GEMM, sampler in its epilogue) draws from
    softmax(z / T): empirical distribution and log-probs of the drawn tokens."""
    torch.manual_seed(9)
    B, D, V = 5, 64, 300
    h, w = bf(B, D), bf(V, D, scale=0.3)
    for T in (1.0, 0.7):
        z = (h.float() @ w.float().t()) / T
        p = torch.softmax(z, -1)
        counts = torch.zeros(B, V, device=DEV)
        step = torch.zeros(1, dtype=torch.int64, device=DEV)
        tok = torch.empty(B, dtype=torch.int64, device=DEV)
        lp = torch.empty(B, device=DEV)
        n = 4000
        for _ in range(n):
            assert C().lmhead_sample_small(h, w, None, 0, 0.0, 0.0, tok, lp, T, 1234, step)
            step += 1
            counts[torch.arange(B, device=DEV), tok] += 1
        torch.cuda.synchronize()
        assert C().device_error() == 0
        assert torch.allclose(lp, torch.log(p.gather(1, tok[:, None]).squeeze(1)), atol=2e-2)
        tv = 0.5 * (counts / n - p).abs().sum(-1)
        assert (tv < 0.08).all(), tv


@pytest.mark.parametrize("M", [1, 7, 16, 33, 64])
@pytest.mark.parametrize("prepared", [False, True])
def test_lmhead_sample_small_large_vocab(M, prepared):
    """Qwen2.5 vocabulary (151936 rows, 1187 tiles over the persistent grid): the drawn token's log-prob
    equals z / T - logsumexp(z / T), and at a temperature of 1e-3 the drawn token is the argmax up to
    bf16 rounding. With ``prepared`` the input is bf16(g * x) plus per-128-column sums of squares of x
    (the split RMSNorm)."""
    torch.manual_seed(M)
    D, V, eps = 1536, 151936, 1e-6
    w = bf(V, D, scale=0.05)
    x = bf(M, D)
    g = (1.0 + 0.1 * torch.randn(D, device=DEV)).to(torch.bfloat16)
    xf = x.float()
    hn = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * g.float()).to(torch.bfloat16)
    if prepared:
        h = (xf * g.float()).to(torch.bfloat16)
        part = torch.zeros(D // 128, 256, device=DEV)
        part[:, :M] = xf.pow(2).view(M, D // 128, 128).sum(-1).t()
        args = (h, w, part, D // 128, float(D), eps)
    else:
        args = (hn, w, None, 0, 0.0, 0.0)
    z = hn.float() @ w.float().t()
    step = torch.full((1,), 7, dtype=torch.int64, device=DEV)
    tok = torch.empty(M, dtype=torch.int64, device=DEV)
    lp = torch.empty(M, device=DEV)
    for T in (1.0, 1e-3):
        assert C().lmhead_sample_small(*args, tok, lp, T, 99, step)
        torch.cuda.synchronize()
        if not prepared:  # the regular 128-row tiling draws with the same rules
            tok2, lp2 = torch.empty_like(tok), torch.empty_like(lp)
            C().lmhead_sample(hn, w, tok2, lp2, T, 99, step)
            torch.cuda.synchronize()
            zt = z / T
            if T == 1.0:
                want2 = zt.gather(1, tok2[:, None]).squeeze(1) - torch.logsumexp(zt, -1)
                assert torch.allclose(lp2, want2, atol=0.05), (lp2, want2)
            else:
                assert (z.gather(1, tok2[:, None]).squeeze(1) >= z.max(-1).values - 0.06).all()
        assert C().device_error() == 0
        zt = z / T
        if T == 1.0:
            want_lp = zt.gather(1, tok[:, None]).squeeze(1) - torch.logsumexp(zt, -1)
            assert torch.allclose(lp, want_lp, atol=0.05), (lp, want_lp)
        else:
            # Gumbel noise spans ~20 units of z / T = 0.02 of z: the winner is the argmax up to rounding
            assert (z.gather(1, tok[:, None]).squeeze(1) >= z.max(-1).values - 0.06).all()


def test_ppo_loss_matches_torch():
    from meshy_b200.backend.batch import Batch
    from meshy_b200.backend.loss import LossConfig, ppo_clip_loss

    torch.manual_seed(10)
    T, n_docs = 500, 6
    doc_ids = torch.randint(0, n_docs + 1, (T,), device=DEV)
    mask = (torch.rand(T, device=DEV) > 0.3).float() * (doc_ids < n_docs).float()
    seg = torch.zeros(n_docs + 1, device=DEV).index_add_(0, doc_ids, mask)
    b = Batch(input_ids=None, labels=None, positions=None, mask=mask, doc_ids=doc_ids,
              advantages=torch.randn(n_docs, device=DEV), rollout_logprobs=-torch.rand(T, device=DEV) * 3,
              cu_seqlens=None, max_seqlen=0, n_docs=n_docs, seg_count=seg,
              positive_lm_weights=torch.rand(n_docs, device=DEV))
    old = -torch.rand(T, device=DEV) * 3
    for cfg in (LossConfig(0.2, 0.28), LossConfig(0.2, 0.2, use_tis=True), LossConfig(0.2, 0.2, use_icepop=True),
                LossConfig(0.2, 0.2, positive_lm_coef=0.1, per_token=True)):
        new = (old + torch.randn(T, device=DEV) * 0.3).requires_grad_(True)
        loss, sums = ppo_clip_loss(new, old, b, 12, 400, cfg, entropy=torch.rand(T, device=DEV))
        loss.backward()
        g_native = new.grad.clone()
        from meshy_b200.ops import functional as Fx

        new2 = new.detach().clone().requires_grad_(True)
        with Fx.torch_baseline():
            loss2, sums2 = ppo_clip_loss(new2, old, b, 12, 400, cfg, entropy=torch.rand(T, device=DEV))
        loss2.backward()
        assert abs(loss.item() - loss2.item()) < 1e-4 + 1e-4 * abs(loss2.item())
        assert rel_err(g_native, new2.grad) < 1e-4
        for k in ("ratio_sum", "clip_sum", "token_count", "ppo_kl_sum", "ess_sum", "train_rollout_kl_sum"):
            assert abs(sums[k].item() - sums2[k].item()) < 1e-3 * (1 + abs(sums2[k].item())), k


def test_adamw_and_norm():
    torch.manual_seed(11)
    n = 100003
    p = torch.randn(n, device=DEV)
    g = torch.randn(n, device=DEV)
    m = torch.zeros(n, device=DEV)
    v = torch.zeros(n, device=DEV)
    out = torch.empty(n, dtype=torch.bfloat16, device=DEV)
    nrm = torch.zeros(1, device=DEV)
    C().sq_norm(g, nrm)
    assert abs(nrm.sqrt().item() - g.norm().item()) < 1e-3 * g.norm().item()
    p2, m2, v2 = p.clone(), m.clone(), v.clone()
    gn = nrm.sqrt()
    C().adamw_flat(p, g, m, v, out, None, gn, 1.0, 1e-3, 0.9, 0.999, 1e-8, 0.1, 1)
    scale = min(1.0, 1.0 / (gn.item() + 1e-6))
    ref.adamw_(p2, g, m2, v2, lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.1, step=1, grad_scale=scale)
    assert torch.allclose(p, p2, atol=1e-6, rtol=1e-5)
    assert torch.equal(out, p.to(torch.bfloat16))


def test_gae_scan_matches_cpu():
    from meshy_b200.backend import gae

    torch.manual_seed(12)
    rows, S = 3, 5000
    mask = torch.zeros(rows, S)
    for r, (a, b) in enumerate([(10, 4000), (0, 5000), (100, 101)]):
        mask[r, a:b] = 1
    doc = torch.arange(rows).unsqueeze(1).expand(rows, S).contiguous()
    rewards = torch.zeros(rows, S)
    rewards[0, 3998] = 1.0
    rewards[1, 4998] = -1.0
    values = torch.randn(rows, S) * 0.1
    adv_cpu, _ = gae.compute_vapo_gae(rewards, values, mask, doc, rows, gamma=1.0, alpha=1.5)
    adv_gpu, _ = gae.compute_vapo_gae(rewards.cuda(), values.cuda(), mask.cuda(), doc.cuda(), rows, gamma=1.0,
                                      alpha=1.5)
    assert torch.allclose(adv_gpu.cpu(), adv_cpu, atol=1e-3)


def test_embedding_fwd_bwd():
    torch.manual_seed(13)
    V, D, T = 1000, 256, 777
    w = bf(V, D)
    ids = torch.randint(0, V, (T,), device=DEV)
    out = torch.empty(T, D, dtype=torch.bfloat16, device=DEV)
    C().embedding_fwd(ids, w, out)
    assert torch.equal(out, w[ids])
    g = bf(T, D)
    gw = torch.zeros(V, D, device=DEV)
    C().embedding_bwd(ids, g, gw)
    ref_gw = torch.zeros(V, D, device=DEV).index_add_(0, ids, g.float())
    assert torch.allclose(gw, ref_gw, atol=1e-4)


# ── small-M (decode) GEMM: swapped operands, cluster split-K through DSMEM ──────────────
@pytest.mark.parametrize("M", [1, 8, 17, 64, 100, 256])
@pytest.mark.parametrize("N,K", [(2048, 1536), (1536, 8960), (1000, 200), (20480, 256)])
def test_gemm_small_m(M, N, K):
    torch.manual_seed(10)
    a, b, bias, res = bf(M, K), bf(N, K), bf(N), bf(M, N)
    out = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    C().gemm(a, b, out, False, False, bias, res, None, 0, False, 0)
    torch.cuda.synchronize()
    assert C().device_error() == 0
    assert rel_err(out, a.float() @ b.float().t() + bias.float() + res.float()) < 1e-2
    out32 = torch.empty(M, N, dtype=torch.float32, device=DEV)
    C().gemm(a, b, out32, False, False, None, None, None, 0, False, 0)
    assert rel_err(out32, a.float() @ b.float().t()) < 5e-3


@pytest.mark.parametrize("cs", [1, 2, 3, 8, 12, 16])
def test_gemm_small_m_cluster_sizes(cs):
    torch.manual_seed(11)
    M, N, K = 48, 1536, 8960
    a, b = bf(M, K), bf(N, K)
    out = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    try:
        C().gemm_small_config(-1, cs)
        C().gemm(a, b, out, False, False, None, None, None, 0, False, 0)
    finally:
        C().gemm_small_config(-1, 0)
    assert rel_err(out, a.float() @ b.float().t()) < 1e-2


@pytest.mark.parametrize("M", [5, 64, 200])
def test_gemm_small_m_swiglu(M):
    torch.manual_seed(12)
    K, N = 1536, 2048
    x, w13 = bf(M, K), bf(N, K, scale=0.05)
    out = torch.empty(M, N // 2, dtype=torch.bfloat16, device=DEV)
    C().gemm(x, w13, out, False, False, None, None, None, 1, False, 64)
    h = (x.float() @ w13.float().t()).to(torch.bfloat16).float().view(M, N // 128, 2, 64)
    want = (torch.nn.functional.silu(h[:, :, 0]) * h[:, :, 1]).reshape(M, N // 2)
    assert rel_err(out, want) < 1e-2
    # same op through the regular tiling must agree
    ref_out = torch.empty_like(out)
    try:
        C().gemm_small_config(0, -1)
        C().gemm(x, w13, ref_out, False, False, None, None, None, 1, False, 64)
    finally:
        C().gemm_small_config(1, -1)
    assert rel_err(out, ref_out) < 1e-2


@pytest.mark.parametrize("splits", [1, 2, 3, 8, 12])
@pytest.mark.parametrize("hd,Hq,Hkv", [(128, 12, 2), (64, 4, 2), (128, 16, 1)])
def test_paged_decode_tma_splits(splits, hd, Hq, Hkv):
    torch.manual_seed(21)
    page, B = 64, 9
    lens = [1, 63, 64, 65, 200, 513, 1000, 1700, 31]
    max_pages = 28
    n_pages = sum((L + page - 1) // page for L in lens) + 3
    kc = bf(n_pages, Hkv, page, hd)
    vc = bf(n_pages, Hkv, page, hd)
    perm = torch.randperm(n_pages, device=DEV)
    bt = torch.zeros(B, max_pages, dtype=torch.int32, device=DEV)
    used = 0
    for b, L in enumerate(lens):
        npg = (L + page - 1) // page
        bt[b, :npg] = perm[used:used + npg].int()
        used += npg
    seq = torch.tensor(lens, dtype=torch.int32, device=DEV)
    q = bf(B, Hq, hd)
    out = torch.empty_like(q)
    try:
        C().paged_decode_force_splits(splits)
        C().paged_attention(q, kc, vc, bt, seq, out, 1 / math.sqrt(hd), None)
    finally:
        C().paged_decode_force_splits(0)
    torch.cuda.synchronize()
    assert C().device_error() == 0
    o_ref = ref.attention_decode_paged(q.float(), kc.float(), vc.float(), bt, seq, 1 / math.sqrt(hd))
    assert rel_err(out, o_ref) < 1e-2


@pytest.mark.parametrize("qk_norm", [False, True])
def test_qkv_rope_cache_matches_rope_then_scatter(qk_norm):
    torch.manual_seed(22)
    T, Hq, Hkv, hd, page, n_pages = 37, 12, 2, 128, 64, 8
    qkv = bf(T, (Hq + 2 * Hkv) * hd)
    pos = torch.randint(0, 4000, (T,), dtype=torch.int32, device=DEV)
    qn = bf(hd) if qk_norm else None
    kn = bf(hd) if qk_norm else None
    slots = torch.randperm(n_pages * page, device=DEV)[:T].long()
    q1, k1, v1 = (torch.empty(T, h, hd, dtype=torch.bfloat16, device=DEV) for h in (Hq, Hkv, Hkv))
    C().qkv_rope_fwd(qkv, pos, qn, kn, q1, k1, v1, 1e4, 1e-6)
    kc1 = torch.zeros(n_pages, Hkv, page, hd, dtype=torch.bfloat16, device=DEV)
    vc1 = torch.zeros_like(kc1)
    C().kv_write(k1, v1, kc1, vc1, slots)
    q2 = torch.empty_like(q1)
    kc2, vc2 = torch.zeros_like(kc1), torch.zeros_like(vc1)
    C().qkv_rope_cache(qkv, pos, qn, kn, q2, None, None, kc2, vc2, slots, 1e4, 1e-6)
    torch.cuda.synchronize()
    assert torch.equal(q1, q2) and torch.equal(kc1, kc2) and torch.equal(vc1, vc2)


@pytest.mark.parametrize("M", [1, 8, 64, 130])
@pytest.mark.parametrize("swiglu", [False, True])
def test_gemm_norm_fused_matches_rmsnorm_then_gemm(M, swiglu):
    torch.manual_seed(23)
    K, N = 1536, 2048
    x, g, w, b = bf(M, K), bf(K), bf(N, K, scale=0.05), bf(N)
    h = torch.empty_like(x)
    rstd = torch.empty(M, device=DEV)
    C().rmsnorm_fwd(x, g, h, rstd, 1e-6)
    n_out = N // 2 if swiglu else N
    want = torch.empty(M, n_out, dtype=torch.bfloat16, device=DEV)
    got = torch.empty_like(want)
    if swiglu:
        C().gemm(h, w, want, False, False, None, None, None, 1, False, 64)
        ok = C().gemm_norm(x, g, 1e-6, w, got, None, None, 1, 64)
    else:
        C().gemm(h, w, want, False, False, b, None, None, 0, False, 0)
        ok = C().gemm_norm(x, g, 1e-6, w, got, b, None, 0, 0)
    torch.cuda.synchronize()
    if M > 128 and swiglu:
        assert not ok  # large-M SwiGLU stays on the regular tiling
        return
    assert ok
    assert C().device_error() == 0
    assert torch.equal(got, want) or rel_err(got, want) < 2e-3


@pytest.mark.parametrize("hd", [64, 128])
def test_flash_attn_chunks_offsets_fwd_bwd(hd):
    """Query chunks at key offsets against separate key documents (the context-parallel form)."""
    from meshy_b200.ops import functional as Fx

    torch.manual_seed(24)
    Hq, Hkv, S, c = 8, 2, 256, 64
    rows = 2
    cu_q = torch.tensor([0, c, 2 * c], dtype=torch.int32, device=DEV)
    cu_k = torch.tensor([0, S, 2 * S], dtype=torch.int32, device=DEV)
    q_off = torch.tensor([64, 192], dtype=torch.int32, device=DEV)
    q = bf(rows * c, Hq, hd).requires_grad_(True)
    k = bf(rows * S, Hkv, hd).requires_grad_(True)
    v = bf(rows * S, Hkv, hd).requires_grad_(True)
    out = Fx.flash_attn_chunks(q, k, v, cu_q, cu_k, q_off, c, S)
    go = bf(*out.shape)
    out.backward(go)
    qr, kr, vr = (t.detach().float().cpu().requires_grad_(True) for t in (q, k, v))
    o_ref = ref.attention_chunks(qr, kr, vr, cu_q.cpu(), cu_k.cpu(), q_off.cpu())
    o_ref.backward(go.float().cpu())
    assert rel_err(out.cpu(), o_ref) < 1e-2
    assert rel_err(q.grad.cpu(), qr.grad) < 3e-2
    assert rel_err(k.grad.cpu(), kr.grad) < 3e-2
    assert rel_err(v.grad.cpu(), vr.grad) < 3e-2
