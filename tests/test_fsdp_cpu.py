"""Sharded parameters (FSDP) on CPU: gloo, 2 ranks.

A trainer whose parameters, gradients and optimiser state are sharded over the DP group must take exactly
the optimiser steps of the replicated data-parallel trainer fed the same samples: several micro-batches
per mini-batch (gradient shards accumulate across them), two mini-batches (gathered blocks go stale after
each step), behaviour log-probs from a no-grad forward, clipping and weight decay, and activation
checkpointing (recompute inside the backward of a gathered block). Its checkpoint restores into a fresh
sharded trainer, and ``full_buffer`` re-assembles the global layout an inference engine loads.
"""

import os
import random
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _samples(rank, seed=0, n=4):
    rng = random.Random(seed * 100 + rank)
    out = []
    for i in range(n):
        # rank 0's short documents share micro-batches, rank 1's long ones do not: unequal micro counts
        P, R = (rng.randint(3, 5), rng.randint(4, 8)) if rank == 0 else (rng.randint(4, 12), rng.randint(56, 70))
        toks = [rng.randrange(2048) for _ in range(P + R)]
        out.append({"tokens": torch.tensor(toks), "mask_assistant": torch.tensor([0] * P + [1] * R),
                    "logprobs": torch.tensor([0.0] * P + [-2.0] * R), "advantage": torch.tensor([1.0 - 0.5 * i]),
                    "reward": torch.tensor([float(i % 2)]), "weight_version": torch.tensor([0])})
    return out


def _trainer(group, fsdp, ckpt_mode="none"):
    from meshy_b200.backend.trainer import PPOTrainer
    from meshy_b200.config import TrainerConfig, TrainerParamsConfig

    tc = TrainerConfig(model_name="qwen3", model_flavor="debugmodel", seq_len=64, lr=1e-3, weight_decay=0.1,
                       max_norm=0.5, dtype="float32", activation_checkpoint_mode=ckpt_mode)
    tp = TrainerParamsConfig(mini_batch_size=2, batch_layout="packed", max_tokens_per_micro=96,
                             old_logprobs_source="train")
    return PPOTrainer(tc, tp, device="cpu", seed=0, dp_group=group, loss_group=group, timer_enabled=False,
                      fsdp_group=group if fsdp else None)


def _worker(rank, world, port, q, tmp):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        g = dist.group.WORLD
        out = {}
        for ckpt_mode in ("none", "full"):
            sh = _trainer(g, True, ckpt_mode)
            rep = _trainer(g, False, ckpt_mode)
            assert sh.flat.numel < rep.flat.numel  # this rank holds about half of the state
            w0 = rep.flat.master.clone()
            for step in range(2):
                m1 = sh.train_step(_samples(rank, step))
                m2 = rep.train_step(_samples(rank, step))
                out[(ckpt_mode, step)] = (m1["grad_norm"], m2["grad_norm"], m1["pg_loss"], m2["pg_loss"])
            # AdamW's first steps move every weight by about lr * sign(g): a gradient that is zero up to rounding
            # can flip sign between the two reduction orders, so compare the updates as a whole
            full = sh.flat.full_buffer("master")
            out[(ckpt_mode, "err")] = float((full - rep.flat.master).norm() / (rep.flat.master - w0).norm())
        # global layout of the gathered weights == the replicated trainer's flat buffer
        full = sh.flat.full_buffer("master")
        sd = sh.flat.state_dict("master")
        out["layout_err"] = max(float((sd[sl.name].reshape(-1) - full[sl.offset:sl.offset + sl.numel]).abs().max())
                                for sl in sh.flat.slots)
        # checkpoint round trip into a fresh sharded trainer
        path = os.path.join(tmp, "ckpt")
        sh.save_checkpoint(path, step=2)
        fresh = _trainer(g, True, "full")
        fresh.load_checkpoint(path)
        out["restore_err"] = max(float((getattr(fresh.flat, n) - getattr(sh.flat, n)).abs().max())
                                 for n in ("master", "exp_avg", "exp_avg_sq"))
        m1 = sh.train_step(_samples(rank, 7))
        m2 = fresh.train_step(_samples(rank, 7))
        out["resume"] = (m1["pg_loss"], m2["pg_loss"], float((sh.flat.master - fresh.flat.master).abs().max()))
        q.put((rank, out))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        import traceback

        q.put((rank, traceback.format_exc()))


@pytest.mark.timeout(600)
def test_sharded_trainer_matches_replicated(tmp_path):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q, str(tmp_path))) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=540) for _ in range(2)]
    for p in ps:
        p.join(timeout=60)
    for rank, out in res:
        assert not isinstance(out, str), out
        for mode in ("none", "full"):
            for step in range(2):
                gn1, gn2, l1, l2 = out[(mode, step)]
                assert abs(gn1 - gn2) <= 1e-5 * max(1.0, gn2), (mode, step, gn1, gn2)
                assert abs(l1 - l2) <= 1e-6 * max(1.0, abs(l2)), (mode, step, l1, l2)
            assert out[(mode, "err")] < 1e-3, (mode, out[(mode, "err")])
        assert out["layout_err"] == 0.0
        assert out["restore_err"] == 0.0
        l1, l2, werr = out["resume"]
        assert l1 == l2 and werr == 0.0
