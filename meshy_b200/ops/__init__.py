"""Hot ops: CUDA kernels on GPU tensors, PyTorch oracle on CPU tensors."""

from . import reference
from .functional import (
    embedding,
    flash_attn_varlen,
    linear,
    linear_swiglu,
    lm_head_logprobs,
    native,
    qkv_rope,
    rmsnorm,
    set_torch_baseline,
    torch_baseline,
)

__all__ = [
    "embedding", "flash_attn_varlen", "linear", "linear_swiglu", "lm_head_logprobs", "native",
    "qkv_rope", "reference", "rmsnorm", "set_torch_baseline", "torch_baseline",
]
