"""L2 prefetch kernels of the decode step (GPU): they launch, change no memory, and a decode with them matches
one without them token for token (same seeds, same weights)."""

import os

import pytest
import torch

pytestmark = pytest.mark.gpu

cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")


@cuda
def test_prefetch_kernels_leave_memory_unchanged():
    from meshy_b200.ops._ext import ext

    C = ext()
    a = torch.randn(3_000_017 // 8 * 8, device="cuda").bfloat16()
    b = torch.randn(1024, 257, device="cuda")
    a0, b0 = a.clone(), b.clone()
    C.l2_prefetch([a, b])
    kc = torch.randn(40, 2, 64, 128, device="cuda").bfloat16()
    vc = torch.randn(40, 2, 64, 128, device="cuda").bfloat16()
    k0, v0 = kc.clone(), vc.clone()
    bt = torch.tensor([[3, 7, 39, -1], [0, 1, 2, 99]], dtype=torch.int32, device="cuda")  # out-of-range ids skipped
    lens = torch.tensor([150, 256], dtype=torch.int32, device="cuda")
    C.kv_prefetch(bt, lens, kc, vc, 64)
    torch.cuda.synchronize()
    assert torch.equal(a, a0) and torch.equal(b, b0) and torch.equal(kc, k0) and torch.equal(vc, v0)


@cuda
@pytest.mark.parametrize("rows", [1, 4])
def test_decode_with_prefetch_matches_without(rows, monkeypatch):
    from meshy_b200.models import build_model, get_model_args
    from meshy_b200.rollout.engine import RolloutEngine

    args = get_model_args("qwen3", "debugmodel")
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, args.vocab_size, (20 + 7 * i,), generator=g).tolist() for i in range(rows)]
    outs = []
    for pf in ("16", "0"):
        monkeypatch.setenv("MESHY_L2_PREFETCH_ROWS", pf)
        eng = RolloutEngine(args, model=build_model(args, seed=0, device="cuda", dtype=torch.bfloat16), max_running=8,
                            max_seq_len=256, device="cuda", seed=5, mem_fraction=0.05)
        gens = eng.generate(prompts, 24, temperature=1.0)
        outs.append([(x.output_ids, [round(v, 4) for v in x.output_logprobs]) for x in gens])
        del eng
        torch.cuda.empty_cache()
    assert outs[0] == outs[1]
