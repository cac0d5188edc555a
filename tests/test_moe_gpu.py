"""Native mixture-of-experts kernels against fp32 PyTorch references (GPU).

* router kernel (softmax + top-k + renormalisation) and its backward against torch autograd;
* the expert layer (device plan + gather, grouped tcgen05 GEMMs, combine) forward and backward against the
  fp32 per-expert loop, including experts that receive no token and weight gradients accumulated into
  ``main_grad``;
* the layer inside a captured CUDA graph (no host synchronisation anywhere in it);
* a whole Qwen3-MoE model: native log-probs and gradients against the PyTorch path.
"""

import math

import pytest
import torch

from meshy_b200.models.moe import moe_experts
from meshy_b200.ops import moe as M

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp_min(1e-12)).item()


def _torch_route(logits, k, norm):
    p = torch.softmax(logits.float(), -1)
    w, e = torch.topk(p, k, dim=-1)
    if norm:
        w = w / w.sum(-1, keepdim=True)
    return w, e


@pytest.mark.parametrize("E,k,norm", [(8, 2, True), (60, 4, False), (128, 8, True), (256, 8, False)])
def test_router_forward_and_backward(E, k, norm):
    torch.manual_seed(E + k)
    T = 513
    logits = (torch.randn(T, E, device=DEV) * 2).to(torch.bfloat16).requires_grad_(True)
    w, e = M.route(logits, k, norm)
    ref = logits.detach().float().requires_grad_(True)
    w_ref, e_ref = _torch_route(ref, k, norm)
    # same experts (as sets per token; torch orders them by value too) and the same weights
    assert torch.equal(e.long().sort(-1).values, e_ref.sort(-1).values)
    order = e.long().argsort(-1)
    order_ref = e_ref.argsort(-1)
    assert torch.allclose(w.gather(-1, order), w_ref.gather(-1, order_ref), atol=1e-5, rtol=1e-4)
    # the upstream gradient is attached to experts, not positions, so tied probabilities (equal bf16 logits)
    # that the two implementations order differently still get the same gradient
    g = torch.randn(T, E, device=DEV)
    w.backward(g.gather(1, e.long()))
    w_ref.backward(g.gather(1, e_ref))
    assert _rel(logits.grad, ref.grad) < 2e-2


def _expert_weights(E, D, F, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    w13 = (torch.randn(E, 2 * F, D, device=DEV, generator=g) / math.sqrt(D)).to(torch.bfloat16)
    w2 = (torch.randn(E, D, F, device=DEV, generator=g) / math.sqrt(F)).to(torch.bfloat16)
    return w13, w2


@pytest.mark.parametrize("T,D,F,E,k", [(300, 256, 128, 8, 2), (1000, 512, 256, 60, 4), (7, 256, 128, 64, 8)])
def test_expert_layer_forward_backward_matches_fp32(T, D, F, E, k):
    torch.manual_seed(T)
    w13, w2 = _expert_weights(E, D, F, T)
    x = torch.randn(T, D, device=DEV).to(torch.bfloat16).requires_grad_(True)
    # a skewed router so that some experts get nothing
    logits = torch.randn(T, E, device=DEV) + torch.linspace(3, -3, E, device=DEV)
    w_ref, e_ref = _torch_route(logits, k, True)
    weights = w_ref.clone().requires_grad_(True)
    experts = e_ref.int()
    w13.main_grad = torch.zeros(w13.shape, dtype=torch.float32, device=DEV)
    w2.main_grad = torch.zeros(w2.shape, dtype=torch.float32, device=DEV)
    out = M.experts_forward(x, weights, experts, w13, w2, 64)
    g = torch.randn(T, D, device=DEV).to(torch.bfloat16)
    out.backward(g)
    torch.cuda.synchronize()
    import meshy_b200._C as C

    assert C.device_error() == 0
    # fp32 oracle: the per-expert loop on fp32 copies
    xr = x.detach().float().requires_grad_(True)
    wr = w_ref.clone().requires_grad_(True)
    w13r = w13.detach().float().requires_grad_(True)
    w2r = w2.detach().float().requires_grad_(True)
    from meshy_b200.ops import functional as Fx

    with Fx.torch_baseline(True):
        ref = moe_experts(xr, wr, e_ref, w13r, w2r, 64)
    ref.backward(g.float())
    assert _rel(out, ref) < 2e-2
    assert _rel(x.grad, xr.grad) < 3e-2
    assert _rel(weights.grad, wr.grad) < 3e-2
    assert _rel(w13.main_grad, w13r.grad) < 3e-2
    assert _rel(w2.main_grad, w2r.grad) < 3e-2


def test_expert_layer_is_graph_capturable():
    torch.manual_seed(0)
    T, D, F, E, k = 6, 256, 128, 32, 4
    w13, w2 = _expert_weights(E, D, F, 5)
    router = (torch.randn(E, D, device=DEV) * 0.1).to(torch.bfloat16)
    x = torch.randn(T, D, device=DEV).to(torch.bfloat16)
    from meshy_b200.ops import functional as Fx

    def step():
        with torch.no_grad():
            w, e = M.route(Fx.linear(x, router), k, True)
            return M.experts_forward(x, w, e, w13, w2, 64)

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        eager = step()
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = step()
    x.copy_(torch.randn(T, D, device=DEV).to(torch.bfloat16))
    graph.replay()
    again = step()
    torch.cuda.synchronize()
    assert _rel(out, again) < 1e-3
    assert _rel(eager, again) > 1e-2  # the replay saw the new input


def test_qwen3_moe_model_native_matches_fp32_torch_path():
    """The whole Qwen3-MoE model: native bf16 log-probs and gradients against the PyTorch path run in fp32 on
    the same weights (the experts chosen by the native router are used on both sides, so near-equal bf16
    router logits cannot send a token to different experts in the two runs)."""
    from meshy_b200.models import build_model, get_model_args
    from meshy_b200.ops import functional as Fx
    import meshy_b200.models.moe as moe_mod

    args = get_model_args("qwen3", "debugmodel_moe")
    torch.manual_seed(0)
    model = build_model(args, seed=0, device=DEV, dtype=torch.bfloat16)
    ref = build_model(args, seed=0, device=DEV, dtype=torch.float32)
    with torch.no_grad():
        for (n, p), (_, q) in zip(model.named_parameters(), ref.named_parameters()):
            q.copy_(p.float())
    lens = [37, 100, 3]
    T = sum(lens)
    ids = torch.randint(0, args.vocab_size, (T,), device=DEV)
    labels = torch.randint(0, args.vocab_size, (T,), device=DEV)
    pos = torch.cat([torch.arange(L, device=DEV) for L in lens]).int()
    cu = torch.tensor([0, 37, 137, 140], dtype=torch.int32, device=DEV)
    picks = []
    real_route = M.route

    def recording_route(logits, k, norm):
        w, e = real_route(logits, k, norm)
        picks.append(e.detach().long())
        return w, e

    mp = pytest.MonkeyPatch()
    mp.setattr(M, "route", recording_route)
    try:
        lp, _ = model.logprobs(ids, labels, pos, cu, max(lens))
        lp.sum().backward()
    finally:
        mp.undo()
    calls = iter(picks)

    def replay_route(x, w_router, top_k, route_norm):
        e = next(calls)
        w = torch.softmax(Fx.linear(x, w_router).float(), -1).gather(-1, e)
        if route_norm:
            w = w / w.sum(-1, keepdim=True)
        return w, e

    mp.setattr(moe_mod, "route", replay_route)
    try:
        with Fx.torch_baseline(True):  # fp32 PyTorch ops on the GPU
            lp_ref, _ = ref.logprobs(ids, labels, pos, cu, max(lens))
            lp_ref.sum().backward()
    finally:
        mp.undo()
    assert _rel(lp, lp_ref) < 2e-2
    for (n, p), (_, q) in zip(model.named_parameters(), ref.named_parameters()):
        assert p.grad is not None and q.grad is not None, n
        assert _rel(p.grad, q.grad) < 6e-2, n


def test_moe_engine_graph_decode_matches_eager():
    """A Qwen3-MoE decode step is captured in a CUDA graph (router, device-side plan and grouped GEMMs, no host
    synchronisation) and replays to the tokens of the eager per-step path."""
    from meshy_b200.models import get_model_args
    from meshy_b200.rollout import RolloutEngine

    args = get_model_args("qwen3", "debugmodel_moe")
    outs = []
    for graph in (False, True):
        e = RolloutEngine(args, device="cuda", max_running=8, max_total_tokens=8192, page_size=64, max_seq_len=512,
                          use_cuda_graph=graph, seed=3, sync_every=4)
        gens = e.generate([[1, 2, 3, 4, 5] * 10, list(range(70)), [9] * 12], [20, 33, 9], temperature=1.0,
                          ignore_eos=True)
        outs.append(gens)
        if graph:
            assert e.stats["graph_replays"] > 0
    for a, b in zip(*outs):
        assert a.output_ids == b.output_ids
        assert max(abs(x - y) for x, y in zip(a.output_logprobs, b.output_logprobs)) < 5e-3


def test_moe_engine_logprobs_match_trainer():
    """The MoE rollout's sampled-token log-probs equal the MoE trainer's recomputed ones (bf16 tolerance)."""
    from meshy_b200.backend.batch import build_micro_batch
    from meshy_b200.backend.plan import MicroPlan
    from meshy_b200.config import TrainerConfig, TrainerParamsConfig
    from meshy_b200.rl import ColocatedGRPO

    tc = TrainerConfig(model_name="qwen3", model_flavor="debugmodel_moe", seq_len=512)
    tp = TrainerParamsConfig(mini_batch_size=4, batch_layout="packed", max_tokens_per_micro=2048,
                             old_logprobs_source="train")
    rl = ColocatedGRPO(tc, tp, device="cuda", group_size=2,
                       engine_kwargs=dict(max_running=8, max_total_tokens=8192, max_seq_len=512, sync_every=4))
    samples = rl.rollout([[5, 6, 7, 8, 9, 10], list(range(40))], 24)
    micro = MicroPlan(tuple(range(len(samples))), 128 * 2, tuple(len(s["tokens"]) for s in samples))
    b = build_micro_batch(samples, micro, layout="packed", device="cuda", need_rollout_lp=True)
    with torch.no_grad():
        lp, _ = rl.trainer.forward_batch(b)
    m = b.mask > 0
    diff = (lp[m] - b.rollout_logprobs[m]).abs()
    assert diff.mean().item() < 0.05, diff.mean()
