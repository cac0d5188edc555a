"""VAPO helpers (reference ``meshy/backend/titan/vapo.py:6-50``).

* :func:`whiten` — global advantage whitening over masked tokens (sums
  all-reduced over the loss group, corrected for context-parallel replicas);
* :func:`clipped_value_error` — PPO-style clipped squared value error
  ``max((V - R)^2, (V_old + clip(V - V_old, -c, c) - R)^2)``;
* :func:`param_groups` — AdamW decay / no-decay split (norm gains, biases and
  the value head bias are not decayed).
"""

from __future__ import annotations

import torch

from .gae import whiten


def clipped_value_error(values: torch.Tensor, returns: torch.Tensor, old_values: torch.Tensor | None,
                        clip: float | None) -> torch.Tensor:
    err = (values - returns) ** 2
    if clip is None or old_values is None:
        return err
    clipped = old_values + (values - old_values).clamp(-clip, clip)
    return torch.maximum(err, (clipped - returns) ** 2)


def param_groups(named_params, weight_decay: float) -> list[dict]:
    decay, no_decay = [], []
    for name, p in named_params:
        if not p.requires_grad:
            continue
        (no_decay if (p.ndim < 2 or name.endswith("bias") or "norm" in name) else decay).append(p)
    groups = []
    if decay:
        groups.append({"params": decay, "weight_decay": weight_decay})
    if no_decay:
        groups.append({"params": no_decay, "weight_decay": 0.0})
    return groups


__all__ = ["clipped_value_error", "param_groups", "whiten"]
