"""HSDP on CPU (gloo, 4 ranks = 2 replicas x 2 shards).

``build_parallel_dims(dp_replicate=2, dp_shard=2)`` gives every rank a shard group (the 2 ranks that split
one replica's parameters) and a replicate group (the 2 ranks that hold the same shard). The sharded trainer
reduce-scatters inside its shard group during backward and all-reduces the gradient shards over the
replicate group before the step; its optimiser steps must equal those of the replicated data-parallel
trainer over all 4 ranks fed the same samples.
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
        P, R = rng.randint(4, 12), rng.randint(6, 40)
        toks = [rng.randrange(2048) for _ in range(P + R)]
        out.append({"tokens": torch.tensor(toks), "mask_assistant": torch.tensor([0] * P + [1] * R),
                    "logprobs": torch.tensor([0.0] * P + [-2.0] * R), "advantage": torch.tensor([1.0 - 0.5 * i]),
                    "reward": torch.tensor([float(i % 2)]), "weight_version": torch.tensor([0])})
    return out


def _trainer(dp, loss, fsdp=None, rep=None):
    from meshy_b200.backend.trainer import PPOTrainer
    from meshy_b200.config import TrainerConfig, TrainerParamsConfig

    tc = TrainerConfig(model_name="qwen3", model_flavor="debugmodel", seq_len=64, lr=1e-3, weight_decay=0.1,
                       max_norm=0.5, dtype="float32")
    tp = TrainerParamsConfig(mini_batch_size=2, batch_layout="packed", max_tokens_per_micro=96,
                             old_logprobs_source="train")
    return PPOTrainer(tc, tp, device="cpu", seed=0, dp_group=dp, loss_group=loss, timer_enabled=False,
                      fsdp_group=fsdp, replicate_group=rep)


def _worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from meshy_b200.parallel.mesh import build_parallel_dims

        pd = build_parallel_dims(world, rank, dp_replicate=2, dp_shard=2)
        assert dist.get_world_size(pd.shard_group) == 2 and dist.get_world_size(pd.replicate_group) == 2
        sh = _trainer(pd.batch_group, pd.loss_group, pd.shard_group, pd.replicate_group)
        rep = _trainer(pd.batch_group, pd.loss_group)
        w0 = rep.flat.master.clone()
        norms = []
        for step in range(2):
            m1 = sh.train_step(_samples(rank, step))
            m2 = rep.train_step(_samples(rank, step))
            norms.append((m1["grad_norm"], m2["grad_norm"]))
        full = sh.flat.full_buffer("master")
        err = float((full - rep.flat.master).norm() / (rep.flat.master - w0).norm())
        q.put((rank, norms, err))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        import traceback

        q.put((rank, traceback.format_exc(), None))


@pytest.mark.timeout(600)
def test_hsdp_matches_replicated_data_parallel():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, 4, port, q)) for r in range(4)]
    for p in ps:
        p.start()
    res = [q.get(timeout=540) for _ in range(4)]
    for p in ps:
        p.join(timeout=60)
    for rank, norms, err in res:
        assert not isinstance(norms, str), norms
        for a, b in norms:
            assert abs(a - b) <= 1e-5 * max(1.0, b), norms
        assert err < 1e-3, err
