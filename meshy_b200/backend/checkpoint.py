"""Trainer / critic state checkpoints in torch DCP format, under torchtitan's keys.

A checkpoint is the DCP directory ``state/{svc}/step-N/`` that the reference's torchtitan checkpointer
writes (``meshy/backend/titan/trainer.py:1080-1089``), with the same key layout, so a run can resume from
the other framework's state:

* model weights (fp32 master) at their torchtitan FQNs, top level (``tok_embeddings.weight``,
  ``layers.0.attention.qkv_linear.wq.weight`` ...; see :mod:`meshy_b200.models.titan_names`);
* AdamW state as PyTorch's flattened optimizer state dict under ``optimizer``:
  ``optimizer.state.<fqn>.exp_avg`` / ``exp_avg_sq`` / ``step`` and ``optimizer.param_groups.<fqn>.lr`` ...;
* ``train_state.step`` / ``train_state.ntokens_seen`` (torchtitan's ``TrainState``).

Writing is sharded: every rank of the data-parallel group writes the parameters it owns (whole
parameters, dealt out by size so each rank writes about 1/world of the bytes) through one collective
``dcp.save``; the AdamW moments of a sharded optimiser and a sharded fp32 master are gathered on the
device first. Loading reads every key on every rank (each rank holds the whole model) and re-shards.
"""

from __future__ import annotations

import os

import torch
import torch.distributed as dist
import torch.distributed.checkpoint as dcp

from ..models.titan_names import join_pieces, titan_pieces


def _group(trainer):
    g = trainer.dp_group
    if g is not None and dist.is_initialized() and dist.get_world_size(g) > 1:
        return g
    return None


def _owners(slots, world: int) -> list[int]:
    """Parameter -> writing rank: largest first onto the least loaded rank (deterministic)."""
    load = [0] * world
    owner = [0] * len(slots)
    for i in sorted(range(len(slots)), key=lambda i: (-slots[i].numel, i)):
        r = min(range(world), key=lambda q: (load[q], q))
        owner[i] = r
        load[r] += slots[i].numel
    return owner


def _moments(trainer):
    """Full-length AdamW moments; an optimiser with sharded moments gathers them (a collective)."""
    f = trainer.flat
    full = getattr(trainer.optimizer, "full_moments", None)
    return full() if full is not None else (f.exp_avg, f.exp_avg_sq)


def _hyper(trainer) -> dict:
    o = trainer.optimizer
    b1, b2 = o.betas
    return {"lr": float(o.lr), "betas": (float(b1), float(b2)), "eps": float(o.eps),
            "weight_decay": float(o.weight_decay), "amsgrad": False, "maximize": False}


def save_trainer_state(trainer, path: str, step: int, ntokens_seen: int = 0) -> None:
    os.makedirs(path, exist_ok=True)
    f = trainer.flat
    args = trainer.model_args
    group = _group(trainer)
    world = dist.get_world_size(group) if group is not None else 1
    rank = dist.get_rank(group) if group is not None else 0
    full = getattr(f, "full_buffer", None)  # sharded parameters: re-assemble the global layout
    if full is not None:
        master, m, v = full("master"), full("exp_avg"), full("exp_avg_sq")
    else:
        f.gather_master()
        master = f.master
        m, v = _moments(trainer)
    owner = _owners(f.slots, world)
    n_steps = torch.tensor(float(trainer.optimizer.step_count))
    hyper = _hyper(trainer)
    sd: dict = {"train_state": {"step": int(step), "ntokens_seen": int(ntokens_seen)},
                "optimizer": {"state": {}, "param_groups": {}}}
    for s, who in zip(f.slots, owner):
        if who != rank:
            continue
        views = [buf[s.offset:s.offset + s.numel].view(s.shape) for buf in (master, m, v)]
        for (fqn, w), (_, a), (_, b) in zip(*(titan_pieces(args, s.name, x) for x in views)):
            sd[fqn] = w.detach().float().cpu().contiguous()
            sd["optimizer"]["state"][fqn] = {"exp_avg": a.detach().float().cpu().contiguous(),
                                             "exp_avg_sq": b.detach().float().cpu().contiguous(),
                                             "step": n_steps.clone()}
            sd["optimizer"]["param_groups"][fqn] = dict(hyper)
    sd["train_state"]["meshy_trainer_step"] = int(trainer.step)
    dcp.save(sd, checkpoint_id=path, process_group=group, no_dist=group is None)


def load_trainer_state(trainer, path: str) -> None:
    f = trainer.flat
    args = trainer.model_args
    group = _group(trainer)
    dev = f.master.device
    sharded = getattr(f, "set_full", None)
    n_full = f.global_numel if sharded is not None else f.numel
    master = torch.zeros(n_full, dtype=torch.float32, device=dev) if sharded is not None else f.master
    moments = (torch.zeros(n_full, dtype=torch.float32, device=dev),
               torch.zeros(n_full, dtype=torch.float32, device=dev))
    # receive buffers for every key (every rank holds the whole model)
    want: dict = {"train_state": {"step": 0, "ntokens_seen": 0, "meshy_trainer_step": 0},
                  "optimizer": {"state": {}}}
    plan = []
    for s in f.slots:
        shape_pieces = titan_pieces(args, s.name, torch.empty(s.shape, device="meta"))
        for fqn, meta in shape_pieces:
            want[fqn] = torch.empty(meta.shape, dtype=torch.float32)
            want["optimizer"]["state"][fqn] = {"exp_avg": torch.empty(meta.shape, dtype=torch.float32),
                                               "exp_avg_sq": torch.empty(meta.shape, dtype=torch.float32),
                                               "step": torch.tensor(0.0)}
        plan.append((s, [fqn for fqn, _ in shape_pieces]))
    dcp.load(want, checkpoint_id=path, process_group=group, no_dist=group is None)
    steps = 0
    with torch.no_grad():
        for s, fqns in plan:
            st = want["optimizer"]["state"]
            master[s.offset:s.offset + s.numel].copy_(join_pieces(args, s.name, [want[q] for q in fqns]).reshape(-1))
            moments[0][s.offset:s.offset + s.numel].copy_(
                join_pieces(args, s.name, [st[q]["exp_avg"] for q in fqns]).reshape(-1))
            moments[1][s.offset:s.offset + s.numel].copy_(
                join_pieces(args, s.name, [st[q]["exp_avg_sq"] for q in fqns]).reshape(-1))
            steps = max(steps, int(float(st[fqns[0]]["step"])))
    opt_sharded = getattr(trainer.optimizer, "set_full_moments", None)
    if sharded is not None:
        sharded("master", master)
        sharded("exp_avg", moments[0])
        sharded("exp_avg_sq", moments[1])
    elif opt_sharded is not None:
        opt_sharded(*moments)
    else:
        f.exp_avg.copy_(moments[0])
        f.exp_avg_sq.copy_(moments[1])
    ts = want["train_state"]
    trainer.step = int(ts.get("meshy_trainer_step") or ts["step"])
    trainer.optimizer.step_count = steps
    f.recast()


__all__ = ["load_trainer_state", "save_trainer_state"]
