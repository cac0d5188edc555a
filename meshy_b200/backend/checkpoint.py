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


def _state(trainer) -> dict:
    f = trainer.flat
    sd = {f"model.{k}": v for k, v in f.state_dict().items()}
    sd.update({f"optim.exp_avg.{s.name}": f.exp_avg[s.offset:s.offset + s.numel].view(s.shape) for s in f.slots})
    sd.update({f"optim.exp_avg_sq.{s.name}": f.exp_avg_sq[s.offset:s.offset + s.numel].view(s.shape)
               for s in f.slots})
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
    sd = {k: v.cpu().clone() for k, v in _state(trainer).items()}
    dcp.load(sd, checkpoint_id=path, no_dist=True)
    live = _state(trainer)
    with torch.no_grad():
        for k, v in live.items():
            if k == "train_state":
                continue
            v.copy_(sd[k])
    trainer.step = int(sd["train_state"][0])
    trainer.optimizer.step_count = int(sd["train_state"][1])
    trainer.flat.recast()


__all__ = ["load_trainer_state", "save_trainer_state"]
