"""Top-K distillation kernels against PyTorch fp32 (GPU).

* ``topk_logprobs`` on given fp32 logits: the same K values and ids as ``torch.topk`` (sorted, largest first)
  and log-probabilities equal to ``value - logsumexp(row)``;
* ``teacher_topk`` (tcgen05 GEMM + select) against the fp32 PyTorch head on the same bf16 weights;
* ``gather_logprobs`` forward and backward (dh and the fp32 main_grad of the weight) against fp32 autograd.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")


def _ext():
    from meshy_b200.ops._ext import ext

    return ext()


@cuda
@pytest.mark.parametrize("V,K", [(50000, 1), (50000, 7), (151936, 64), (4096, 1000)])
def test_topk_logprobs_matches_torch(V, K):
    g = torch.Generator(device="cuda").manual_seed(V + K)
    T = 37
    if K >= 1000:  # distinct values, so the order among the K is unambiguous
        z = torch.stack([torch.randperm(V, device="cuda", generator=g) for _ in range(T)]).float() * 1e-3 - 2.0
    else:
        z = torch.randn(T, V, device="cuda", generator=g) * 4
    z[3] = z[3] - z[3].max() - 1.0  # an all-negative row
    ids = torch.empty(T, K, dtype=torch.long, device="cuda")
    lp = torch.empty(T, K, dtype=torch.float32, device="cuda")
    lse = torch.empty(T, dtype=torch.float32, device="cuda")
    _ext().topk_logprobs(z, K, ids, lp, lse)
    ref = z.double().topk(K, dim=-1)
    ref_lse = torch.logsumexp(z.double(), -1)
    assert torch.equal(ids, ref.indices)
    assert torch.allclose(lse.double(), ref_lse, atol=1e-5, rtol=1e-6)
    assert torch.allclose(lp.double(), ref.values - ref_lse[:, None], atol=2e-5, rtol=1e-6)


@cuda
def test_teacher_topk_matches_fp32_head():
    from meshy_b200.backend.topk_loss import teacher_topk

    g = torch.Generator(device="cuda").manual_seed(1)
    T, D, V, K = 300, 256, 8192, 16
    h = (torch.randn(T, D, device="cuda", generator=g)).bfloat16()
    w = (torch.randn(V, D, device="cuda", generator=g) * 0.05).bfloat16()
    ids, lps = teacher_topk(h, w, K, chunk=128)
    z = h.float() @ w.float().t()
    ref = z.topk(K, dim=-1)
    ref_lp = ref.values - torch.logsumexp(z, -1, keepdim=True)
    assert torch.allclose(lps, ref_lp, atol=2e-3, rtol=0)
    # ids agree except where two candidates are closer than the GEMM's rounding
    assert (ids == ref.indices).float().mean() > 0.98
    # the log-probability of every returned id is that id's log-probability under the fp32 head
    got = z.gather(-1, ids) - torch.logsumexp(z, -1, keepdim=True)
    assert torch.allclose(lps, got, atol=2e-3, rtol=0)


@cuda
@pytest.mark.parametrize("main_grad", [False, True])
def test_gather_logprobs_forward_backward(main_grad):
    from meshy_b200.backend.topk_loss import gather_logprobs

    g = torch.Generator(device="cuda").manual_seed(2)
    T, D, V, K = 520, 256, 6144, 8
    h0 = torch.randn(T, D, device="cuda", generator=g).bfloat16()
    w0 = (torch.randn(V, D, device="cuda", generator=g) * 0.05).bfloat16()
    ids = torch.randint(0, V, (T, K), device="cuda", generator=g)
    ids[5, 3] = ids[5, 1]  # a repeated id within a row
    up = torch.randn(T, K, device="cuda", generator=g)

    h = h0.clone().requires_grad_(True)
    w = w0.clone().requires_grad_(True)
    if main_grad:
        w.main_grad = torch.zeros(V, D, dtype=torch.float32, device="cuda")
    lp = gather_logprobs(h, w, ids, chunk=256)
    (lp * up).sum().backward()

    hr = h0.float().requires_grad_(True)
    wr = w0.float().requires_grad_(True)
    z = hr @ wr.t()
    lpr = z.gather(-1, ids) - torch.logsumexp(z, -1, keepdim=True)
    (lpr * up).sum().backward()

    assert torch.allclose(lp, lpr.detach(), atol=2e-3, rtol=0)
    gw = w.main_grad if main_grad else w.grad.float()
    for got, want in ((h.grad.float(), hr.grad), (gw, wr.grad)):
        err = (got - want).norm() / want.norm()
        assert err < 1e-2, float(err)
