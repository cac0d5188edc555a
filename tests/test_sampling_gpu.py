"""Filtered sampling kernel (top-k / top-p / temperature over fp32 logits) against PyTorch (GPU).

* greedy and top-k 1 pick the argmax; a tiny top-p keeps only the most likely token;
* every draw lies in the kept set of the PyTorch filter (top-k ``z < kth`` masking, top-p on the sorted
  cumulative mass), and its log-probability is the log-softmax of the filtered, tempered logits;
* the empirical distribution over many draws matches the filtered distribution;
* through ``ops.decode.sample`` (tcgen05 logits + the kernel), capturable in a CUDA graph.
"""

import pytest
import torch

import meshy_b200._C as C
from meshy_b200.ops import decode as D
from meshy_b200.ops import reference as R

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _run(logits, temperature, top_k, top_p, seed=0, step=None):
    B = logits.shape[0]
    tok = torch.empty(B, dtype=torch.int64, device=DEV)
    lp = torch.empty(B, dtype=torch.float32, device=DEV)
    C.filtered_sample(logits, temperature, top_k, top_p, seed, step, tok, lp)
    return tok, lp


def _kept(logits, temperature, top_k, top_p):
    z = logits.float() / temperature
    if top_k > 0:
        kth = torch.topk(z, top_k, -1).values[..., -1:]
        z = z.masked_fill(z < kth, float("-inf"))
    if top_p < 1.0:
        sz, idx = torch.sort(z, -1, descending=True)
        p = torch.softmax(sz, -1)
        drop = (p.cumsum(-1) - p) > top_p
        sz = sz.masked_fill(drop, float("-inf"))
        z = torch.full_like(z, float("-inf")).scatter(-1, idx, sz)
    return z


def test_degenerate_filters_pick_the_argmax():
    torch.manual_seed(0)
    logits = torch.randn(7, 5000, device=DEV) * 3
    best = logits.argmax(-1)
    for t, k, p in ((0.0, -1, 1.0), (1.0, 1, 1.0), (0.7, -1, 1e-6)):
        tok, lp = _run(logits, t, k, p)
        assert torch.equal(tok, best), (t, k, p)


@pytest.mark.parametrize("t,k,p", [(1.0, 20, 1.0), (0.8, -1, 0.9), (1.3, 50, 0.7), (1.0, 3000, 0.95)])
def test_draws_stay_in_the_kept_set_with_exact_logprobs(t, k, p):
    torch.manual_seed(1)
    logits = torch.randn(16, 4099, device=DEV) * 2
    z = _kept(logits, t, k, p)
    logp = torch.log_softmax(z, -1)
    step = torch.zeros(1, dtype=torch.int64, device=DEV)
    for s in range(20):
        step.fill_(s)
        tok, lp = _run(logits, t, k, p, seed=5, step=step)
        assert torch.isfinite(z.gather(1, tok[:, None])).all(), "drew a filtered-out token"
        assert torch.allclose(lp, logp.gather(1, tok[:, None]).squeeze(1), atol=1e-4)


def test_empirical_distribution_matches():
    torch.manual_seed(2)
    V = 64
    logits = torch.randn(1, V, device=DEV).repeat(4096, 1)
    tok, _ = _run(logits, 1.0, 10, 0.9, seed=11)
    z = _kept(logits[:1], 1.0, 10, 0.9)
    want = torch.softmax(z, -1)[0]
    got = torch.bincount(tok, minlength=V).float() / tok.numel()
    assert (got - want).abs().max().item() < 0.03
    assert got[torch.isinf(z[0])].sum().item() == 0


def test_decode_sample_path_and_graph_capture():
    torch.manual_seed(3)
    h = torch.randn(4, 256, device=DEV).to(torch.bfloat16)
    w = (torch.randn(3000, 256, device=DEV) * 0.1).to(torch.bfloat16)
    step = torch.zeros(1, dtype=torch.int64, device=DEV)
    tok, lp = D.sample(h, w, 1.0, top_k=40, top_p=0.9, seed=3, step=step)
    z = _kept(R.linear(h.float(), w.float()) if hasattr(R, "linear") else h.float() @ w.float().t(), 1.0, 40, 0.9)
    assert torch.isfinite(z.gather(1, tok[:, None])).all()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        D.sample(h, w, 1.0, top_k=40, top_p=0.9, seed=3, step=step)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        tok_g, lp_g = D.sample(h, w, 1.0, top_k=40, top_p=0.9, seed=3, step=step)
    draws = []
    for i in range(4):
        step.fill_(100 + i)
        g.replay()
        draws.append(tok_g.clone())
    torch.cuda.synchronize()
    assert all(torch.isfinite(z.gather(1, d[:, None])).all() for d in draws)
    assert len({tuple(d.tolist()) for d in draws}) > 1  # the step counter changes the noise
