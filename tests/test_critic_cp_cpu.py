"""Critic under context parallelism (CPU, gloo, 2 ranks): every row of a window is split head-tail over the CP
group, attention runs exactly over the full rows, the values come back whole, and the window loss, the values
and the updated weights equal a single-process critic on the same window (reference behaviour:
``meshy/backend/titan/critic/engine.py:561-618``, CP-aware value training with gathered values)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _critic(cp_group=None, loss_group=None):
    from meshy_b200.backend.critic.trainer import CriticTrainer
    from meshy_b200.models import get_model_args

    args = get_model_args("qwen3", "debugmodel")
    return CriticTrainer(args, device="cpu", lr=1e-3, warmup_steps=0, max_norm=1.0, seq_len=128,
                         max_tokens_per_micro=256, optimizer_kwargs={"weight_decay": 0.01}, seed=0,
                         cp_group=cp_group, loss_group=loss_group)


def _window():
    from meshy_b200.backend.critic.data import TrajectorySample

    g = torch.Generator().manual_seed(4)
    out = []
    for i in range(3):
        n = 17 + 9 * i
        mask = [0.0] * 5 + [1.0] * (n - 5)
        out.append(TrajectorySample(tokens=torch.randint(0, 2048, (n,), generator=g).tolist(), mask=mask,
                                    reward=float(i % 2)))
    return out


def _worker(rank, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=2)
        c = _critic(cp_group=dist.group.WORLD, loss_group=dist.group.WORLD)
        w = _window()
        loss, values, _ = c.train_window(w, [0, 1, 2])
        pred = c.predict(w, [0, 1, 2])
        q.put((rank, loss, {k: v.numpy().copy() for k, v in values.items()},
               {k: v.numpy().copy() for k, v in pred.items()}, c.flat.master.numpy().copy()))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        import traceback

        q.put((rank, traceback.format_exc(), None, None, None))


@pytest.mark.timeout(300)
def test_cp_critic_matches_single_rank():
    ref = _critic()
    w = _window()
    loss_ref, values_ref, _ = ref.train_window(w, [0, 1, 2])
    pred_ref = ref.predict(w, [0, 1, 2])
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=240) for _ in range(2)]
    for p in ps:
        p.join(timeout=60)
    for rank, loss, values, pred, master in res:
        assert not isinstance(loss, str), loss
        assert loss == pytest.approx(loss_ref, rel=1e-5, abs=1e-7)
        for r in range(3):
            assert torch.allclose(torch.from_numpy(values[r]), values_ref[r], atol=1e-5), r
            assert torch.allclose(torch.from_numpy(pred[r]), pred_ref[r], atol=1e-5), r
        assert torch.allclose(torch.from_numpy(master), ref.flat.master, atol=1e-6)
