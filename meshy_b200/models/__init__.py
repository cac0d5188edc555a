"""Model families: architecture registry, decoder module, HF checkpoint mapping."""

from .args import ModelArgs, MoEArgs, get_model_args, list_models
from .transformer import Block, DecoderLM, build_model

__all__ = ["Block", "DecoderLM", "ModelArgs", "MoEArgs", "build_model", "get_model_args", "list_models"]
