"""MiniCPM5: registry scalars and numerical parity with HF ``LlamaForCausalLM`` (CPU, fp32).

The registry must carry MiniCPM5's published architecture (1B and 2B). For numerics no checkpoint can be
downloaded here, so a randomly initialised HF Llama model with MiniCPM5's layout (GQA with 2 KV heads, a
head_dim that is not dim / n_heads, RoPE theta 5e6, untied head) is built at a small width, its HF state
dict is loaded through this package's HF mapping, and the fp32 logits of both models must agree; the
mapping must also round-trip (export then import gives the same tensors).
"""

import dataclasses

import pytest
import torch

from meshy_b200.models import build_model, get_model_args
from meshy_b200.models.hf import from_hf, to_hf


@pytest.mark.parametrize("flavor,dim,layers,ffn", [("1B", 1536, 24, 4608), ("2B", 2048, 42, 6144)])
def test_registry_matches_published_architecture(flavor, dim, layers, ffn):
    a = get_model_args("minicpm5", flavor)
    assert (a.dim, a.n_layers, a.ffn_dim) == (dim, layers, ffn)
    assert (a.n_heads, a.n_kv_heads, a.head_dim) == (16, 2, 128)
    assert a.vocab_size == 130560 and not a.tie_embeddings and not a.qkv_bias and not a.qk_norm
    assert a.rope_theta == 5e6 and a.norm_eps == 1e-6 and a.max_seq_len == 131072
    assert a.q_dim == 2048 and a.kv_dim == 256  # head_dim is 128 even where dim / n_heads is 96


def _small():
    # MiniCPM5-1B's shape ratios at a CPU size: head_dim (64) != dim / n_heads (48)
    return dataclasses.replace(get_model_args("minicpm5", "1B"), dim=384, n_layers=2, n_heads=8, head_dim=64,
                               ffn_dim=256, vocab_size=512)


def test_logits_match_hf_llama():
    from transformers import LlamaConfig, LlamaForCausalLM

    a = _small()
    cfg = LlamaConfig(hidden_size=a.dim, num_hidden_layers=a.n_layers, num_attention_heads=a.n_heads,
                      num_key_value_heads=a.n_kv_heads, head_dim=a.head_dim, intermediate_size=a.ffn_dim,
                      vocab_size=a.vocab_size, rope_theta=a.rope_theta, rms_norm_eps=a.norm_eps,
                      tie_word_embeddings=False, max_position_embeddings=4096, attention_bias=False,
                      mlp_bias=False)
    torch.manual_seed(0)
    hf = LlamaForCausalLM(cfg).float().eval()
    ours = build_model(a, seed=1, device="cpu", dtype=torch.float32).eval()
    sd = from_hf(a, {k: v for k, v in hf.state_dict().items()})
    with torch.no_grad():
        for name, p in ours.named_parameters():
            p.copy_(sd[name])
    ids = torch.randint(0, a.vocab_size, (1, 37))
    with torch.no_grad():
        want = hf(input_ids=ids).logits[0]
        got = ours.logits(ids[0], torch.arange(37, dtype=torch.int32), torch.tensor([0, 37], dtype=torch.int32), 37)
    assert torch.allclose(got.float(), want, atol=2e-4, rtol=1e-4), (got - want).abs().max()
    assert torch.equal(got.argmax(-1), want.argmax(-1))


def test_hf_mapping_round_trip():
    a = _small()
    model = build_model(a, seed=2, device="cpu", dtype=torch.float32)
    sd = {n: p.detach() for n, p in model.named_parameters()}
    back = from_hf(a, to_hf(a, sd, dtype=torch.float32))
    assert set(back) == set(sd)
    for n in sd:
        assert torch.equal(back[n], sd[n]), n
