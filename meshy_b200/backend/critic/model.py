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


class _ValueHeadLoss(torch.autograd.Function):
    """Fused value head + clipped value loss on the native kernels (``value_head_fwd`` / ``value_head_bwd``)."""

    @staticmethod
    def forward(ctx, h, w, b, returns, mask, old, clip, denom):
        from ...ops._ext import ext

        C = ext()
        T = h.shape[0]
        v = torch.empty(T, dtype=torch.float32, device=h.device)
        dv = torch.empty(T, dtype=torch.float32, device=h.device)
        num = torch.zeros(1, dtype=torch.float32, device=h.device)
        C.value_head_fwd(h.contiguous(), w.reshape(-1).float().contiguous(), b.reshape(-1).float().contiguous(),
                         returns.float().contiguous(), mask.float().contiguous(),
                         None if old is None else old.float().contiguous(), float(clip or 0.0), 1.0 / float(denom),
                         v, dv, num)
        ctx.save_for_backward(h, w, dv)
        ctx.mark_non_differentiable(v)
        return num[0] / float(denom), v

    @staticmethod
    def backward(ctx, gloss, _gv):
        from ...ops._ext import ext

        h, w, dv = ctx.saved_tensors
        dv = (dv * gloss.float()).contiguous()
        dh = torch.empty_like(h)
        dw = torch.zeros(w.numel(), dtype=torch.float32, device=h.device)
        db = torch.zeros(1, dtype=torch.float32, device=h.device)
        ext().value_head_bwd(h.contiguous(), w.reshape(-1).float().contiguous(), dv, dh, dw, db)
        return dh, dw.view_as(w), db, None, None, None, None, None


def value_head_loss(h, w, b, returns, mask, old=None, clip=None, denom: float = 1.0):
    """``(loss, values)``: ``loss = sum(mask * clipped_err(h w + b, returns, old)) / denom`` with gradients for
    ``h``, ``w`` and ``b``; ``values`` (fp32, detached) are the head's outputs. Native kernels for bf16 CUDA
    hidden states, PyTorch otherwise."""
    from ...ops.functional import native
    from ..vapo import clipped_value_error

    if native(h) and h.dtype == torch.bfloat16:
        return _ValueHeadLoss.apply(h, w, b, returns, mask, old, clip, denom)
    v = (h.float() @ w.t()).squeeze(-1) + b
    err = clipped_value_error(v, returns, old, clip) * mask
    return err.sum() / denom, v.detach()


__all__ = ["CriticModel", "critic_args_from_actor", "value_head_loss"]
