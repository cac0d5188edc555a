"""Trainer / critic state checkpoints in torch DCP format.

Layout matches the reference's global checkpoint shard (``state/{svc}/step-N/``
DCP directory, written collectively; ``meshy/backend/titan/trainer.py:1080-1089``).
The state is the flat fp32 master weights (by parameter name), the AdamW
moments and step, and the trainer step counter.
"""

from __future__ import annotations

import os

import torch
import torch.distributed as dist
import torch.distributed.checkpoint as dcp


def _moments(trainer):
    """Full-length AdamW moments; an optimiser with sharded moments gathers them (a collective)."""
    f = trainer.flat
    full = getattr(trainer.optimizer, "full_moments", None)
    return full() if full is not None else (f.exp_avg, f.exp_avg_sq)


def _state(trainer, moments=None) -> dict:
    f = trainer.flat
    m, v = moments if moments is not None else _moments(trainer)
    sd = {f"model.{k}": t for k, t in f.state_dict().items()}
    sd.update({f"optim.exp_avg.{s.name}": m[s.offset:s.offset + s.numel].view(s.shape) for s in f.slots})
    sd.update({f"optim.exp_avg_sq.{s.name}": v[s.offset:s.offset + s.numel].view(s.shape) for s in f.slots})
    sd["train_state"] = torch.tensor([trainer.step, trainer.optimizer.step_count], dtype=torch.int64)
    return sd


def save_trainer_state(trainer, path: str, step: int) -> None:
    os.makedirs(path, exist_ok=True)
    sd = _state(trainer)
    # every DP replica holds the full state; rank 0 of the group writes it
    if dist.is_initialized() and trainer.dp_group is not None and dist.get_world_size(trainer.dp_group) > 1:
        if dist.get_rank(trainer.dp_group) == 0:
            dcp.save({k: v.cpu() for k, v in sd.items()}, checkpoint_id=path, no_dist=True)
        dist.barrier(trainer.dp_group)
    else:
        dcp.save({k: v.cpu() for k, v in sd.items()}, checkpoint_id=path, no_dist=True)


def load_trainer_state(trainer, path: str) -> None:
    f = trainer.flat
    sharded = getattr(trainer.optimizer, "set_full_moments", None)
    # full-length moment buffers to load into (the live ones when the optimiser keeps them whole)
    moments = ((torch.zeros(f.numel, dtype=torch.float32, device=f.master.device),
                torch.zeros(f.numel, dtype=torch.float32, device=f.master.device)) if sharded is not None
               else (f.exp_avg, f.exp_avg_sq))
    live = _state(trainer, moments)
    sd = {k: v.cpu().clone() for k, v in live.items()}
    dcp.load(sd, checkpoint_id=path, no_dist=True)
    with torch.no_grad():
        for k, v in live.items():
            if k == "train_state":
                continue
            v.copy_(sd[k])
    if sharded is not None:
        sharded(*moments)
    trainer.step = int(sd["train_state"][0])
    trainer.optimizer.step_count = int(sd["train_state"][1])
    trainer.flat.recast()


__all__ = ["load_trainer_state", "save_trainer_state"]
