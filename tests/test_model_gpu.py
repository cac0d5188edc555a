"""End-to-end native-kernel paths vs the PyTorch path on the same weights (GPU)."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


@pytest.mark.parametrize("model", [("qwen3", "debugmodel"), ("qwen2_5_math", "R1-Distill-1.5B")])
def test_forward_backward_native_vs_torch(model):
    from meshy_b200.backend.flat import FlatParams
    from meshy_b200.models import build_model, get_model_args
    from meshy_b200.ops import functional as Fx

    args = get_model_args(*model)
    if args.n_layers > 4:
        from dataclasses import replace

        args = replace(args, n_layers=2)
    dev = torch.device("cuda")
    m = build_model(args, seed=0, device=dev, dtype=torch.float32)
    flat = FlatParams(m, compute_dtype=torch.bfloat16, device=dev)
    lens = [37, 128, 300, 64]
    T = sum(lens)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32, device=dev)
    ids = torch.randint(0, args.vocab_size, (T,), device=dev)
    labels = torch.roll(ids, -1)
    pos = torch.cat([torch.arange(L, dtype=torch.int32) for L in lens]).to(dev)
    lp, ent = m.logprobs(ids, labels, pos, cu, max(lens), with_entropy=True)
    g = torch.randn(T, device=dev)
    flat.zero_grad()
    (lp * g).sum().backward()
    grad_native = flat.grad.clone()
    with Fx.torch_baseline():
        flat.zero_grad()
        for p in flat.params:
            p.grad = None
        lp2, ent2 = m.logprobs(ids, labels, pos, cu, max(lens), with_entropy=True)
        (lp2 * g).sum().backward()
        grad_torch = torch.zeros_like(flat.grad)
        for s, p in zip(flat.slots, flat.params):
            if p.grad is not None:
                grad_torch[s.offset:s.offset + s.numel] = p.grad.float().reshape(-1)
    assert torch.allclose(lp, lp2, atol=0.1, rtol=0.02), (lp - lp2).abs().max()
    assert _rel(ent, ent2) < 2e-2
    assert _rel(grad_native, grad_torch) < 0.05


def test_engine_graph_decode_matches_eager():
    from meshy_b200.models import get_model_args
    from meshy_b200.rollout import RolloutEngine

    args = get_model_args("qwen3", "debugmodel")
    outs = []
    for graph in (False, True):
        e = RolloutEngine(args, device="cuda", max_running=8, max_total_tokens=8192, page_size=64, max_seq_len=512,
                          use_cuda_graph=graph, seed=3, sync_every=4)
        gens = e.generate([[1, 2, 3, 4, 5] * 10, list(range(70))], [20, 33], temperature=1.0, ignore_eos=True)
        outs.append(gens)
    for a, b in zip(*outs):
        assert a.output_ids == b.output_ids
        assert len(a.output_ids) in (20, 33)
        # the graph path pads the batch to its bucket, which changes the GEMM tiling and split-K
        # summation order; bf16 re-rounding of the hidden state then moves logprobs by ~1e-3
        assert max(abs(x - y) for x, y in zip(a.output_logprobs, b.output_logprobs)) < 5e-3


def test_engine_logprobs_match_trainer():
    """The rollout's sampled-token log-probs equal the trainer's recomputed ones (bf16 tolerance)."""
    from meshy_b200.config import TrainerConfig, TrainerParamsConfig
    from meshy_b200.rl import ColocatedGRPO

    tc = TrainerConfig(model_name="qwen3", model_flavor="debugmodel", seq_len=512)
    tp = TrainerParamsConfig(mini_batch_size=4, batch_layout="packed", max_tokens_per_micro=2048,
                             old_logprobs_source="train")
    rl = ColocatedGRPO(tc, tp, device="cuda", group_size=2,
                       engine_kwargs=dict(max_running=8, max_total_tokens=8192, max_seq_len=512, sync_every=4))
    samples = rl.rollout([[5, 6, 7, 8, 9, 10], list(range(40))], 24)
    from meshy_b200.backend.batch import build_micro_batch
    from meshy_b200.backend.plan import MicroPlan

    micro = MicroPlan(tuple(range(len(samples))), 128 * 2, tuple(len(s["tokens"]) for s in samples))
    b = build_micro_batch(samples, micro, layout="packed", device="cuda", need_rollout_lp=True)
    with torch.no_grad():
        lp, _ = rl.trainer.forward_batch(b)
    m = b.mask > 0
    diff = (lp[m] - b.rollout_logprobs[m]).abs()
    assert diff.mean().item() < 0.05, diff.mean()


def test_engine_release_resume_keeps_addresses_and_graphs():
    """Colocation hand-off through virtual-memory regions: physical pages go back to the driver, the
    addresses (and so the captured decode graphs) survive, weights come back bit-exact."""
    from meshy_b200.models import get_model_args
    from meshy_b200.rollout import RolloutEngine

    args = get_model_args("qwen3", "debugmodel")
    e = RolloutEngine(args, device="cuda", max_running=8, max_total_tokens=1 << 16, page_size=64, max_seq_len=512,
                      use_cuda_graph=True, seed=3, sync_every=4)
    e.generate([[1, 2, 3, 4, 5] * 4], [12], ignore_eos=True)
    n_graphs = len(e._graphs)
    w_before = e.weight_flat.clone()
    kv_ptr, w_ptr = e.kv.data_ptr(), e.weight_flat.data_ptr()
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    e.release_memory()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 - free0 >= e.kv.numel() * 2  # at least the KV cache went back
    assert all(e.memory_released.values())
    with pytest.raises(RuntimeError, match="released"):
        e.update_weights_from_flat(w_before)
    e.resume_memory()
    assert e.kv.data_ptr() == kv_ptr and e.weight_flat.data_ptr() == w_ptr
    assert torch.equal(e.weight_flat, w_before)
    gens = e.generate([[1, 2, 3, 4, 5] * 4, [7, 8, 9]], [12, 9], ignore_eos=True)
    assert [len(g.output_ids) for g in gens] == [12, 9]
    assert len(e._graphs) >= n_graphs
