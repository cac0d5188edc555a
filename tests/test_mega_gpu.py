"""The whole-step persistent decode kernel vs the per-op decode path on the same engine state (GPU).

Both paths start from the same prefilled KV cache and decode state; the kernel's final hidden states
and the K/V rows it writes for the step must match the per-op path's to bf16 accuracy (the two paths
round intermediate values at slightly different points and sum split-K partials in different orders).
"""

import random

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _enable(monkeypatch):
    monkeypatch.setenv("MESHY_MEGA", "1")


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


def _args(kind: str):
    from meshy_b200.models import get_model_args
    from meshy_b200.models.args import ModelArgs

    if kind == "r1":
        return get_model_args("qwen2_5_math", "R1-Distill-1.5B")
    qk = kind == "qknorm"
    return ModelArgs(name="qwen3" if qk else "qwen2_5", flavor="mega_test", dim=512, n_layers=3, n_heads=8,
                     n_kv_heads=2, head_dim=128, ffn_dim=1024, vocab_size=4096, rope_theta=1e6, qk_norm=qk,
                     qkv_bias=not qk, max_seq_len=8192)


def _prefilled(args, lens, seed=0):
    from meshy_b200.rollout import RolloutEngine

    e = RolloutEngine(args, device="cuda", max_running=64, max_total_tokens=1 << 18, page_size=64,
                      max_seq_len=8192, use_cuda_graph=False, seed=seed, sync_every=4,
                      prefill_chunk_tokens=1 << 20)
    assert e._mega is not None, e.mega_reason
    rng = random.Random(seed)
    for L in lens:
        e.submit([rng.randrange(args.vocab_size) for _ in range(L)], 16, ignore_eos=True)
    e._admit()
    assert len(e.running) == len(lens)
    e._ensure_pages(range(len(lens)), 2)
    return e


def _compare(e):
    from meshy_b200.ops._ext import ext

    n = len(e.running)
    kv0 = e.kv.clone()
    h_ref = e._decode_hidden_layers(n).clone()
    kv_ref = e.kv.clone()
    e.kv.copy_(kv0)
    ext().clear_device_error()
    h = e._mega(e.st, n).clone()
    torch.cuda.synchronize()
    err = int(ext().device_error())
    if err:
        words = e._mega.ws[9][2048:2064].tolist()
        ext().clear_device_error()
        e._mega.reset()
        raise AssertionError(f"device error {err}; barrier/exit/debug words {words}")
    assert torch.isfinite(h.float()).all()
    assert _rel(h, h_ref) < 2e-2, _rel(h, h_ref)
    written = (kv_ref != kv0).any(-1)  # rows of this step's K/V
    assert written.any()
    assert _rel(e.kv[written], kv_ref[written]) < 2e-2
    assert torch.equal(e.kv[~written], kv0[~written])  # nothing else touched
    return h


@pytest.mark.parametrize("kind", ["bias", "qknorm"])
@pytest.mark.parametrize("lens", [[5], [3000], [70, 1, 129, 640, 64], [900] * 16, [300 + 37 * i for i in range(40)]])
def test_mega_decode_matches_per_op(kind, lens):
    _compare(_prefilled(_args(kind), lens))


def test_mega_decode_r1_distill_b64():
    lens = [200 + 31 * i for i in range(64)]
    _compare(_prefilled(_args("r1"), lens))


def test_mega_decode_in_cuda_graph():
    e = _prefilled(_args("bias"), [100, 700, 1300])
    n = len(e.running)
    h_eager = e._mega(e.st, n).clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        out = e._mega(e.st, n)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    # split-K partial sums are added with float atomics, so run-to-run sums differ in their last bits
    assert _rel(out[:n], h_eager) < 1e-2


def test_mega_engine_generate_runs_long():
    """Many consecutive steps through the engine (graphs on): the counters and accumulators stay
    consistent from launch to launch and the outputs stay finite."""
    from meshy_b200.ops._ext import ext
    from meshy_b200.rollout import RolloutEngine

    args = _args("bias")
    e = RolloutEngine(args, device="cuda", max_running=64, max_total_tokens=1 << 18, page_size=64,
                      max_seq_len=4096, use_cuda_graph=True, seed=1, sync_every=8)
    assert e._mega is not None
    gens = e.generate([[1 + i, 2, 3] * (5 + i) for i in range(24)], [100 + 7 * i for i in range(24)],
                      temperature=1.0, ignore_eos=True)
    torch.cuda.synchronize()
    assert int(ext().device_error()) == 0
    for i, gen in enumerate(gens):
        assert len(gen.output_ids) == 100 + 7 * i
        assert all(lp <= 0.0 and lp == lp for lp in gen.output_logprobs)
