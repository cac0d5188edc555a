"""Tensor parallelism on CPU (gloo, 2 ranks): column/row-split blocks with all-reduces give the same loss
and the same (re-assembled) gradient as the unsplit model."""

import os
import random
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _samples():
    rng = random.Random(5)
    out = []
    for i in range(4):
        P, R = rng.randint(4, 10), rng.randint(6, 20)
        out.append({"tokens": torch.tensor([rng.randrange(2048) for _ in range(P + R)]),
                    "mask_assistant": torch.tensor([0] * P + [1] * R),
                    "logprobs": torch.tensor([0.0] * P + [-2.0] * R), "advantage": torch.tensor([1.0 - 0.5 * i]),
                    "reward": torch.tensor([float(i % 2)]), "weight_version": torch.tensor([0])})
    return out


def _trainer(tp_group=None):
    from meshy_b200.backend.trainer import PPOTrainer
    from meshy_b200.config import TrainerConfig, TrainerParamsConfig

    tc = TrainerConfig(model_name="qwen3", model_flavor="debugmodel", seq_len=64, lr=1e-3, weight_decay=0.0,
                       max_norm=0.0, dtype="float32", tp_degree=2 if tp_group is not None else 1)
    tp = TrainerParamsConfig(mini_batch_size=4, batch_layout="packed", max_tokens_per_micro=512,
                             old_logprobs_source="train")
    return PPOTrainer(tc, tp, device="cpu", seed=0, tp_group=tp_group, timer_enabled=False)


def _worker(rank, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=2)
        t = _trainer(dist.group.WORLD)
        m = t.train_step(_samples())
        q.put((rank, {s.name: t.flat.view(t.flat.grad, s.name).numpy().copy() for s in t.flat.slots}, m["pg_loss"]))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        import traceback

        q.put((rank, traceback.format_exc(), None))


@pytest.mark.timeout(300)
def test_tensor_parallel_step_matches_single_rank():
    ref = _trainer()
    m = ref.train_step(_samples())
    want = {s.name: ref.flat.view(ref.flat.grad, s.name) for s in ref.flat.slots}
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
    parts = {}
    for rank in range(2):
        _, grads, loss = res[rank]
        assert not isinstance(grads, str), grads
        assert abs(loss - m["pg_loss"]) < 1e-4 * max(1.0, abs(m["pg_loss"]))
        parts[rank] = {k: torch.from_numpy(v) for k, v in grads.items()}
    from meshy_b200.models import get_model_args

    a = get_model_args("qwen3", "debugmodel")
    hd, H, Hk = a.head_dim, a.n_heads, a.n_kv_heads
    for name, w in want.items():
        g0, g1 = parts[0][name], parts[1][name]
        if name.endswith(".wqkv"):
            q0, k0, v0 = g0.split([H // 2 * hd, Hk // 2 * hd, Hk // 2 * hd])
            q1, k1, v1 = g1.split([H // 2 * hd, Hk // 2 * hd, Hk // 2 * hd])
            got = torch.cat([q0, q1, k0, k1, v0, v1])
        elif name.endswith(".wo") or name.endswith(".w2"):
            got = torch.cat([g0, g1], 1)
        elif name.endswith(".w13"):
            got = torch.cat([g0, g1])
        else:
            assert torch.allclose(g0, g1, atol=1e-6), name  # replicated parameters agree across TP ranks
            got = g0
        err = ((got - w).norm() / w.norm().clamp_min(1e-12)).item()
        assert err < 1e-4, (name, err)
