"""Critic network: the actor's decoder backbone plus a scalar fp32 value head.

Same structure as the reference (``meshy/backend/titan/critic/model.py:40-187``):
the backbone is the actor architecture up to the final norm (no LM head, so
no weight tying), loaded from the same base weights; the value head
``V_t = h_t · w + b`` is fp32 and zero-initialised so a cold critic predicts 0
for every state and its first gradient comes only from the returns.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from ..gae import ADVANTAGE_TOKENS  # noqa: F401 (re-export for callers)
from ...models.args import ModelArgs
from ...models.transformer import build_model


def critic_args_from_actor(args: ModelArgs) -> ModelArgs:
    """The critic shares every architecture scalar with its actor (no LM head)."""
    return args


class CriticModel(nn.Module):
    def __init__(self, args: ModelArgs, *, seed: int = 0, device="cpu", backbone: nn.Module | None = None):
        super().__init__()
        self.args = args
        self.backbone = backbone if backbone is not None else build_model(
            args, seed=seed, device=device, dtype=torch.float32, with_lm_head=False)
        self.value_head = nn.Parameter(torch.zeros(1, args.dim, dtype=torch.float32, device=device))
        self.value_bias = nn.Parameter(torch.zeros(1, dtype=torch.float32, device=device))

    def backbone_parameters(self):
        return self.backbone.named_parameters()

    def forward(self, input_ids, positions, cu_seqlens, max_seqlen) -> torch.Tensor:
        """Per-token values ``[T]`` (fp32) of a packed token stream."""
        h = self.backbone.hidden(input_ids, positions, cu_seqlens, max_seqlen)
        return (h.float() @ self.value_head.t()).squeeze(-1) + self.value_bias


__all__ = ["CriticModel", "critic_args_from_actor"]
