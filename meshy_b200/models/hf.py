"""HF checkpoint mapping (safetensors) for every family.

Maps this package's fused parameter layout to HF names and back:
``wqkv`` ↔ ``q_proj/k_proj/v_proj`` (+ biases), ``w13`` ↔ ``gate_proj`` /
``up_proj`` (block-interleaved), MoE ``w13[e]`` ↔ ``experts.e.*``.  Reference
counterparts: ``meshy/backend/titan/models/qwen2_5/state_dict_adapter.py:25-43``
and ``minicpm5/state_dict_adapter.py:33-61`` (which also undo torchtitan's
interleaved-RoPE row permutation; not needed here because the model uses the
HF rotate-half convention natively).
"""

from __future__ import annotations

import json
import os

import torch

from ..ops.reference import interleave_w13, split_w13
from .args import ModelArgs


def to_hf(args: ModelArgs, sd: dict[str, torch.Tensor], dtype=torch.bfloat16) -> dict[str, torch.Tensor]:
    out: dict[str, torch.Tensor] = {}
    q, kv = args.q_dim, args.kv_dim
    cvt = lambda t: t.detach().to(dtype).contiguous()  # noqa: E731
    out["model.embed_tokens.weight"] = cvt(sd["embed"])
    out["model.norm.weight"] = cvt(sd["norm"])
    if "lm_head" in sd:
        out["lm_head.weight"] = cvt(sd["lm_head"])
    for i in range(args.n_layers):
        p, h = f"layers.{i}.", f"model.layers.{i}."
        w = sd[p + "wqkv"]
        out[h + "self_attn.q_proj.weight"] = cvt(w[:q])
        out[h + "self_attn.k_proj.weight"] = cvt(w[q:q + kv])
        out[h + "self_attn.v_proj.weight"] = cvt(w[q + kv:])
        if p + "bqkv" in sd:
            b = sd[p + "bqkv"]
            out[h + "self_attn.q_proj.bias"] = cvt(b[:q])
            out[h + "self_attn.k_proj.bias"] = cvt(b[q:q + kv])
            out[h + "self_attn.v_proj.bias"] = cvt(b[q + kv:])
        if p + "q_norm" in sd:
            out[h + "self_attn.q_norm.weight"] = cvt(sd[p + "q_norm"])
            out[h + "self_attn.k_norm.weight"] = cvt(sd[p + "k_norm"])
        out[h + "self_attn.o_proj.weight"] = cvt(sd[p + "wo"])
        out[h + "input_layernorm.weight"] = cvt(sd[p + "attn_norm"])
        out[h + "post_attention_layernorm.weight"] = cvt(sd[p + "mlp_norm"])
        if args.moe is None:
            g, u = split_w13(sd[p + "w13"], args.swiglu_block)
            out[h + "mlp.gate_proj.weight"] = cvt(g)
            out[h + "mlp.up_proj.weight"] = cvt(u)
            out[h + "mlp.down_proj.weight"] = cvt(sd[p + "w2"])
        else:
            out[h + "mlp.gate.weight"] = cvt(sd[p + "moe.router"])
            w13, w2 = sd[p + "moe.w13"], sd[p + "moe.w2"]
            for e in range(w13.shape[0]):
                g, u = split_w13(w13[e], args.swiglu_block)
                out[h + f"mlp.experts.{e}.gate_proj.weight"] = cvt(g)
                out[h + f"mlp.experts.{e}.up_proj.weight"] = cvt(u)
                out[h + f"mlp.experts.{e}.down_proj.weight"] = cvt(w2[e])
    return out


def from_hf(args: ModelArgs, hf: dict[str, torch.Tensor]) -> dict[str, torch.Tensor]:
    sd: dict[str, torch.Tensor] = {"embed": hf["model.embed_tokens.weight"], "norm": hf["model.norm.weight"]}
    if not args.tie_embeddings:
        sd["lm_head"] = hf.get("lm_head.weight", hf["model.embed_tokens.weight"])
    for i in range(args.n_layers):
        p, h = f"layers.{i}.", f"model.layers.{i}."
        sd[p + "wqkv"] = torch.cat([hf[h + f"self_attn.{n}_proj.weight"] for n in "qkv"], 0)
        if args.qkv_bias:
            sd[p + "bqkv"] = torch.cat([hf[h + f"self_attn.{n}_proj.bias"] for n in "qkv"], 0)
        if args.qk_norm:
            sd[p + "q_norm"] = hf[h + "self_attn.q_norm.weight"]
            sd[p + "k_norm"] = hf[h + "self_attn.k_norm.weight"]
        sd[p + "wo"] = hf[h + "self_attn.o_proj.weight"]
        sd[p + "attn_norm"] = hf[h + "input_layernorm.weight"]
        sd[p + "mlp_norm"] = hf[h + "post_attention_layernorm.weight"]
        if args.moe is None:
            sd[p + "w13"] = interleave_w13(hf[h + "mlp.gate_proj.weight"], hf[h + "mlp.up_proj.weight"],
                                           args.swiglu_block)
            sd[p + "w2"] = hf[h + "mlp.down_proj.weight"]
        else:
            E = args.moe.n_experts
            sd[p + "moe.router"] = hf[h + "mlp.gate.weight"]
            sd[p + "moe.w13"] = torch.stack([
                interleave_w13(hf[h + f"mlp.experts.{e}.gate_proj.weight"], hf[h + f"mlp.experts.{e}.up_proj.weight"],
                               args.swiglu_block) for e in range(E)])
            sd[p + "moe.w2"] = torch.stack([hf[h + f"mlp.experts.{e}.down_proj.weight"] for e in range(E)])
    return sd


def hf_config(args: ModelArgs) -> dict:
    arch = {"qwen2_5": "Qwen2ForCausalLM", "qwen2_5_math": "Qwen2ForCausalLM", "qwen3": "Qwen3ForCausalLM",
            "minicpm5": "LlamaForCausalLM", "llama3": "LlamaForCausalLM"}[args.name]
    if args.moe is not None:
        arch = "Qwen3MoeForCausalLM"
    cfg = {
        "architectures": [arch], "hidden_size": args.dim, "num_hidden_layers": args.n_layers,
        "num_attention_heads": args.n_heads, "num_key_value_heads": args.n_kv_heads, "head_dim": args.head_dim,
        "intermediate_size": args.ffn_dim, "vocab_size": args.vocab_size, "rope_theta": args.rope_theta,
        "rms_norm_eps": args.norm_eps, "tie_word_embeddings": args.tie_embeddings,
        "max_position_embeddings": args.max_seq_len, "torch_dtype": "bfloat16",
        "meshy_b200": {"model_name": args.name, "flavor": args.flavor},
    }
    if args.moe is not None:
        cfg.update({"num_experts": args.moe.n_experts, "num_experts_per_tok": args.moe.top_k,
                    "moe_intermediate_size": args.moe.expert_ffn_dim, "norm_topk_prob": args.moe.route_norm})
    return cfg


def save_hf_checkpoint(args: ModelArgs, sd: dict[str, torch.Tensor], output_dir: str) -> str:
    from safetensors.torch import save_file

    os.makedirs(output_dir, exist_ok=True)
    path = os.path.join(output_dir, "model.safetensors")
    hf = {k: v.cpu() for k, v in to_hf(args, sd).items()}
    save_file(hf, path + ".tmp")
    os.replace(path + ".tmp", path)
    with open(os.path.join(output_dir, "config.json"), "w") as f:
        json.dump(hf_config(args), f, indent=1)
    return path


def load_hf_checkpoint(args: ModelArgs, path: str) -> dict[str, torch.Tensor]:
    from safetensors.torch import load_file

    if os.path.isdir(path):
        files = sorted(f for f in os.listdir(path) if f.endswith(".safetensors"))
        hf: dict[str, torch.Tensor] = {}
        for f in files:
            hf.update(load_file(os.path.join(path, f)))
    else:
        hf = load_file(path)
    return from_hf(args, hf)


__all__ = ["from_hf", "hf_config", "load_hf_checkpoint", "save_hf_checkpoint", "to_hf"]
