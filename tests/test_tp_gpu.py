"""Tensor-parallel training on 2 GPUs (one process per GPU, NCCL): the column/row-split blocks give the loss of
the unsplit model and, slice by slice, its gradient (bf16 tolerance), on the native kernels."""

import os
import random
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _samples():
    rng = random.Random(5)
    out = []
    for i in range(4):
        P, R = rng.randint(16, 40), rng.randint(40, 120)
        out.append({"tokens": torch.tensor([rng.randrange(2048) for _ in range(P + R)]),
                    "mask_assistant": torch.tensor([0] * P + [1] * R),
                    "logprobs": torch.tensor([0.0] * P + [-2.0] * R), "advantage": torch.tensor([1.0 - 0.5 * i]),
                    "reward": torch.tensor([float(i % 2)]), "weight_version": torch.tensor([0])})
    return out


def _trainer(device, tp_group=None):
    from meshy_b200.backend.trainer import PPOTrainer
    from meshy_b200.config import TrainerConfig, TrainerParamsConfig

    tc = TrainerConfig(model_name="qwen3", model_flavor="debugmodel", seq_len=256, lr=1e-3, weight_decay=0.0,
                       max_norm=0.0, dtype="bfloat16", tp_degree=2 if tp_group is not None else 1)
    tp = TrainerParamsConfig(mini_batch_size=4, batch_layout="packed", max_tokens_per_micro=1024,
                             old_logprobs_source="train")
    return PPOTrainer(tc, tp, device=device, seed=0, tp_group=tp_group, timer_enabled=False)


def _grads(t):
    return {s.name: t.flat.view(t.flat.grad, s.name).float().cpu().clone() for s in t.flat.slots}


def _worker(rank, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        from datetime import timedelta

        dist.init_process_group("nccl", rank=rank, world_size=2, device_id=torch.device("cuda", rank),
                                timeout=timedelta(seconds=120))
        t = _trainer(f"cuda:{rank}", dist.group.WORLD)
        m = t.train_step(_samples())
        q.put((rank, _grads(t), m["pg_loss"]))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        import traceback

        q.put((rank, traceback.format_exc(), None))


def _rel(a, b):
    return float((a - b).norm() / b.norm().clamp_min(1e-12))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.timeout(300)
def test_tensor_parallel_training_on_two_gpus_matches_unsplit():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = {r[0]: r for r in (q.get(timeout=240) for _ in range(2))}
    for p in ps:
        p.join(timeout=60)
    for r in range(2):
        assert not isinstance(res[r][1], str), res[r][1]
    ref = _trainer("cuda:0")
    m = ref.train_step(_samples())
    want = _grads(ref)
    from meshy_b200.models import get_model_args
    from meshy_b200.parallel.tp import tp_shard_param

    a = get_model_args("qwen3", "debugmodel")
    for r in range(2):
        _, grads, loss = res[r]
        assert abs(loss - m["pg_loss"]) < 1e-2 * max(1.0, abs(m["pg_loss"]))
        for name, full in want.items():
            part = tp_shard_param(name, full, a, 2, r)
            assert _rel(grads[name], part) < 5e-2, (r, name, _rel(grads[name], part))
