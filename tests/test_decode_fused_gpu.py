"""Decode with RMSNorm split across GEMMs vs the unfused per-op decode, same engine state (GPU).

The residual GEMMs (o_proj, down_proj) also write bf16(g * x) and per-tile sums of squares; the
consuming GEMMs (QKV, gate/up) scale their rows by rstd; optionally the QKV GEMM's epilogue also
applies RoPE (+ QK-norm) and writes K/V into the paged cache. The hidden states of one decode step
and the K/V rows it writes must match the unfused path to bf16 accuracy.
"""

import random

import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


@pytest.mark.parametrize("model,lens", [
    (("qwen2_5_math", "R1-Distill-1.5B"), [5, 300, 1000]),
    (("qwen2_5_math", "R1-Distill-1.5B"), [64 + 7 * i for i in range(40)]),
    (("qwen3", "1.7B"), [100, 2000]),
    (("minicpm5", "1B"), [33] * 8),
])
@pytest.mark.parametrize("fused_rope", [0, 1])
def test_split_norm_decode_matches_unfused(model, lens, fused_rope, monkeypatch):
    from dataclasses import replace

    from meshy_b200.models import get_model_args
    from meshy_b200.rollout import RolloutEngine

    args = replace(get_model_args(*model), n_layers=4)
    e = RolloutEngine(args, device="cuda", max_running=64, max_total_tokens=1 << 17, page_size=64, max_seq_len=4096,
                      use_cuda_graph=False, seed=0, prefill_chunk_tokens=1 << 20)
    rng = random.Random(0)
    for L in lens:
        e.submit([rng.randrange(args.vocab_size) for _ in range(L)], 8, ignore_eos=True)
    e._admit()
    n = len(e.running)
    e._ensure_pages(range(n), 2)
    kv0 = e.kv.clone()
    from meshy_b200.ops._ext import ext

    monkeypatch.setenv("MESHY_SPLIT_NORM", "0")
    monkeypatch.setenv("MESHY_FUSED_QKV_ROPE", str(fused_rope))
    c0 = ext().launch_count()
    h_ref = e._decode_hidden_layers(n).clone()
    launches_ref = ext().launch_count() - c0
    kv_ref = e.kv.clone()
    e.kv.copy_(kv0)
    monkeypatch.setenv("MESHY_SPLIT_NORM", "1")
    c0 = ext().launch_count()
    h = e._decode_hidden_layers(n).clone()
    launches = ext().launch_count() - c0
    torch.cuda.synchronize()
    assert _rel(h, h_ref) < 2e-2, _rel(h, h_ref)
    assert _rel(e.kv, kv_ref) < 2e-2
    # every norm between the first and the final one is folded into the GEMMs
    L = len(e.model.layers)
    # RoPE + KV write ride on the QKV GEMM of every layer after the first
    assert launches_ref - launches == 2 * L - 1 + (L - 1) * fused_rope, (launches_ref, launches)
