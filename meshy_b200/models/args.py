"""Architecture descriptions and the flavor registry.

One dataclass, :class:`ModelArgs`, describes every decoder family the
framework trains and serves.  The registry maps the ``(model_name,
model_flavor)`` pair a :class:`~meshy_b200.config.TrainerConfig` names to an
instance, mirroring the reference's torchtitan model specs:

* ``qwen2_5`` / ``qwen2_5_math``: Qwen2 blocks with QKV bias, no QK-norm
  (reference ``meshy/backend/titan/models/qwen2_5/__init__.py:148-439`` and
  ``qwen2_5_math/__init__.py:50-160``; R1-Distill-1.5B at ``:84-98``).
* ``qwen3``: QK-norm, no bias; dense flavors and the 30B-A3B MoE (torchtitan's
  in-tree ``qwen3`` spec that the reference imports).
* ``minicpm5``: Llama block, GQA kv=2, head_dim 128, RoPE theta 5e6
  (reference ``meshy/backend/titan/models/minicpm5/__init__.py:64-189``).
* ``llama3``: plain Llama-3 blocks (torchtitan in-tree).

RoPE convention: every family uses the rotate-half pairing (dims ``i`` and
``i + head_dim/2``), which is the HF checkpoint convention, so HF weights load
without the row permutation torchtitan's interleaved complex RoPE needs.
"""

from __future__ import annotations

from dataclasses import dataclass, field, replace


@dataclass(frozen=True)
class MoEArgs:
    n_experts: int
    top_k: int
    expert_ffn_dim: int
    #: renormalise the selected top-k router weights to sum to one
    route_norm: bool = True
    #: "softmax" scores over all experts, then top-k (Qwen3-MoE)
    score_func: str = "softmax"
    n_shared_experts: int = 0


@dataclass(frozen=True)
class ModelArgs:
    name: str
    flavor: str
    dim: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    ffn_dim: int
    vocab_size: int
    rope_theta: float = 1e4
    qkv_bias: bool = False
    qk_norm: bool = False
    tie_embeddings: bool = False
    norm_eps: float = 1e-6
    max_seq_len: int = 131072
    moe: MoEArgs | None = None
    #: block size of the gate/up interleave in the fused ``w13`` weight.  Row
    #: block ``2i`` holds gate rows ``[i*G, (i+1)*G)``, block ``2i+1`` the
    #: matching up rows, so one GEMM output tile carries both halves of every
    #: SwiGLU pair and the activation runs in the GEMM epilogue.
    swiglu_block: int = 64

    @property
    def q_dim(self) -> int:
        return self.n_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_dim

    @property
    def qkv_dim(self) -> int:
        return self.q_dim + 2 * self.kv_dim

    def num_params(self, include_embedding: bool = True) -> int:
        d, L = self.dim, self.n_layers
        attn = d * self.qkv_dim + self.q_dim * d + (self.qkv_dim if self.qkv_bias else 0)
        if self.qk_norm:
            attn += 2 * self.head_dim
        if self.moe is None:
            mlp = 3 * d * self.ffn_dim
        else:
            mlp = self.moe.n_experts * 3 * d * self.moe.expert_ffn_dim + self.moe.n_experts * d
            mlp += self.moe.n_shared_experts * 3 * d * self.moe.expert_ffn_dim
        per_layer = attn + mlp + 2 * d
        total = L * per_layer + d
        if include_embedding:
            total += self.vocab_size * d * (1 if self.tie_embeddings else 2)
        elif not self.tie_embeddings:
            total += self.vocab_size * d
        return total

    def active_params(self) -> int:
        """Parameters touched per token (MoE counts only top-k experts)."""
        if self.moe is None:
            return self.num_params(include_embedding=False)
        d, L = self.dim, self.n_layers
        attn = d * self.qkv_dim + self.q_dim * d
        mlp = (self.moe.top_k + self.moe.n_shared_experts) * 3 * d * self.moe.expert_ffn_dim
        lm = 0 if self.tie_embeddings else self.vocab_size * d
        return L * (attn + mlp) + lm

    def kv_bytes_per_token(self, dtype_bytes: int = 2) -> int:
        return 2 * self.kv_dim * self.n_layers * dtype_bytes


def _qwen2(flavor, dim, n_layers, n_heads, n_kv, ffn, vocab, tie, theta=1e6, max_seq=131072, name="qwen2_5"):
    return ModelArgs(name=name, flavor=flavor, dim=dim, n_layers=n_layers, n_heads=n_heads,
                     n_kv_heads=n_kv, head_dim=dim // n_heads, ffn_dim=ffn, vocab_size=vocab,
                     rope_theta=theta, qkv_bias=True, qk_norm=False, tie_embeddings=tie,
                     max_seq_len=max_seq)


def _qwen3(flavor, dim, n_layers, n_heads, n_kv, ffn, vocab=151936, tie=False, head_dim=128, moe=None):
    return ModelArgs(name="qwen3", flavor=flavor, dim=dim, n_layers=n_layers, n_heads=n_heads,
                     n_kv_heads=n_kv, head_dim=head_dim, ffn_dim=ffn, vocab_size=vocab,
                     rope_theta=1e6, qkv_bias=False, qk_norm=True, tie_embeddings=tie, moe=moe,
                     max_seq_len=131072)


def _minicpm5(flavor, dim, n_layers, n_heads, ffn):
    return ModelArgs(name="minicpm5", flavor=flavor, dim=dim, n_layers=n_layers, n_heads=n_heads,
                     n_kv_heads=2, head_dim=128, ffn_dim=ffn, vocab_size=130560, rope_theta=5e6,
                     qkv_bias=False, qk_norm=False, tie_embeddings=False, max_seq_len=131072)


def _llama3(flavor, dim, n_layers, n_heads, n_kv, ffn, vocab=128256, theta=5e5):
    return ModelArgs(name="llama3", flavor=flavor, dim=dim, n_layers=n_layers, n_heads=n_heads,
                     n_kv_heads=n_kv, head_dim=dim // n_heads, ffn_dim=ffn, vocab_size=vocab,
                     rope_theta=theta, norm_eps=1e-5)


_REGISTRY: dict[str, dict[str, ModelArgs]] = {
    "qwen2_5": {
        "0.5B": _qwen2("0.5B", 896, 24, 14, 2, 4864, 151936, True),
        "1.5B": _qwen2("1.5B", 1536, 28, 12, 2, 8960, 151936, True),
        "3B": _qwen2("3B", 2048, 36, 16, 2, 11008, 151936, True),
        "7B": _qwen2("7B", 3584, 28, 28, 4, 18944, 152064, False),
    },
    "qwen2_5_math": {
        "Math-1.5B": _qwen2("Math-1.5B", 1536, 28, 12, 2, 8960, 151936, True, 1e4, 4096, "qwen2_5_math"),
        "Math-7B": _qwen2("Math-7B", 3584, 28, 28, 4, 18944, 152064, False, 1e4, 4096, "qwen2_5_math"),
        "R1-Distill-1.5B": _qwen2("R1-Distill-1.5B", 1536, 28, 12, 2, 8960, 151936, False, 1e4, 131072,
                                  "qwen2_5_math"),
        "R1-Distill-7B": _qwen2("R1-Distill-7B", 3584, 28, 28, 4, 18944, 152064, False, 1e4, 131072,
                                "qwen2_5_math"),
    },
    "qwen3": {
        # the CPU oracle decoder.
        "debugmodel": ModelArgs(name="qwen3", flavor="debugmodel", dim=256, n_layers=2, n_heads=4,
                                n_kv_heads=2, head_dim=64, ffn_dim=512, vocab_size=2048, rope_theta=1e6,
                                qk_norm=True, max_seq_len=4096),
        "debugmodel_moe": ModelArgs(name="qwen3", flavor="debugmodel_moe", dim=256, n_layers=2, n_heads=4,
                                    n_kv_heads=2, head_dim=64, ffn_dim=512, vocab_size=2048, rope_theta=1e6,
                                    qk_norm=True, max_seq_len=4096,
                                    moe=MoEArgs(n_experts=8, top_k=2, expert_ffn_dim=128)),
        "0.6B": _qwen3("0.6B", 1024, 28, 16, 8, 3072, tie=True),
        "1.7B": _qwen3("1.7B", 2048, 28, 16, 8, 6144, tie=True),
        "4B": _qwen3("4B", 2560, 36, 32, 8, 9728, tie=True),
        "8B": _qwen3("8B", 4096, 36, 32, 8, 12288),
        "14B": _qwen3("14B", 5120, 40, 40, 8, 17408),
        "32B": _qwen3("32B", 5120, 64, 64, 8, 25600),
        "30B-A3B": _qwen3("30B-A3B", 2048, 48, 32, 4, 6144,
                          moe=MoEArgs(n_experts=128, top_k=8, expert_ffn_dim=768)),
    },
    "minicpm5": {
        "1B": _minicpm5("1B", 1536, 24, 16, 4608),
        "2B": _minicpm5("2B", 2048, 42, 16, 6144),
    },
    "llama3": {
        "debugmodel": ModelArgs(name="llama3", flavor="debugmodel", dim=256, n_layers=2, n_heads=4,
                                n_kv_heads=2, head_dim=64, ffn_dim=512, vocab_size=2048, rope_theta=5e5),
        "8B": _llama3("8B", 4096, 32, 32, 8, 14336),
    },
}


def get_model_args(model_name: str, flavor: str, **overrides) -> ModelArgs:
    """Resolve ``(model_name, flavor)``; ``overrides`` replace fields (tests)."""
    if model_name not in _REGISTRY:
        raise ValueError(f"unknown model {model_name!r}; available: {sorted(_REGISTRY)}")
    flavors = _REGISTRY[model_name]
    if flavor not in flavors:
        raise ValueError(f"unknown {model_name} flavor {flavor!r}; available: {sorted(flavors)}")
    args = flavors[flavor]
    return replace(args, **overrides) if overrides else args


def list_models() -> dict[str, list[str]]:
    return {k: sorted(v) for k, v in _REGISTRY.items()}


__all__ = ["ModelArgs", "MoEArgs", "get_model_args", "list_models"]
