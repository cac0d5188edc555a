"""Expert parallelism on CPU (gloo, 2 ranks): dispatch/combine all-to-all around the local experts equals
the single-process MoE layer on the union of the ranks' tokens, forward and backward."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _layer(seed=0):
    from meshy_b200.models import get_model_args
    from meshy_b200.models.moe import MoE

    args = get_model_args("qwen3", "debugmodel_moe")
    torch.manual_seed(seed)
    m = MoE(args)
    m.reset_parameters(0.05, 0.05)
    return args, m


def _inputs(args):
    g = torch.Generator().manual_seed(7)
    return [torch.randn(11 + 3 * r, args.dim, generator=g) for r in range(2)]


def _worker(rank, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=2)
        from meshy_b200.parallel.ep import shard_experts

        args, moe = _layer()

        class _M(torch.nn.Module):
            def __init__(self):
                super().__init__()
                self.layers = torch.nn.ModuleList([torch.nn.Module()])
                self.layers[0].moe = moe

        shard_experts(_M(), dist.group.WORLD)
        x = _inputs(args)[rank].requires_grad_(True)
        y = moe(x)
        y.pow(2).sum().backward()
        # numpy copies: tensors sent through a Queue are shared memory that dies with this process
        q.put((rank, y.detach().numpy().copy(), x.grad.numpy().copy(), moe.w13.grad.numpy().copy(),
               moe.expert_offset))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        import traceback

        q.put((rank, traceback.format_exc(), None, None, None))


@pytest.mark.timeout(300)
def test_expert_parallel_matches_dense_moe():
    args, moe = _layer()
    xs = [x.clone().requires_grad_(True) for x in _inputs(args)]
    ys = [moe(x) for x in xs]
    sum(y.pow(2).sum() for y in ys).backward()
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
    E_local = moe.w13.shape[0] // 2
    for rank in range(2):
        _, y, gx, gw, off = res[rank]
        assert not isinstance(y, str), y
        y, gx, gw = torch.from_numpy(y), torch.from_numpy(gx), torch.from_numpy(gw)
        assert torch.allclose(y, ys[rank].detach(), atol=1e-5), (y - ys[rank]).abs().max()
        assert torch.allclose(gx, xs[rank].grad, atol=1e-5)
        assert off == rank * E_local
        assert torch.allclose(gw, moe.w13.grad[off:off + E_local], atol=1e-5)


def _trainer_worker(rank, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=2)
        t = _moe_trainer(ep_group=dist.group.WORLD)
        samples = _moe_samples()
        plan = t.plan_batch(samples, 2)
        t.train_step(plan.local_samples(samples, rank), plan=plan.per_rank[rank])
        names = [s.name for s in t.flat.slots]
        q.put((rank, {n: t.flat.view(t.flat.grad, n).numpy().copy() for n in names}))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        import traceback

        q.put((rank, traceback.format_exc()))


def _moe_trainer(ep_group=None, mini: int = 2):
    from meshy_b200.backend.trainer import PPOTrainer
    from meshy_b200.config import TrainerConfig, TrainerParamsConfig

    tc = TrainerConfig(model_name="qwen3", model_flavor="debugmodel_moe", seq_len=64, lr=1e-3, weight_decay=0.0,
                       max_norm=0.05, dtype="float32", ep_degree=2 if ep_group is not None else 1)
    tp = TrainerParamsConfig(mini_batch_size=mini, batch_layout="packed", max_tokens_per_micro=512,
                             old_logprobs_source="train")
    return PPOTrainer(tc, tp, device="cpu", seed=0, dp_group=ep_group, ep_group=ep_group, timer_enabled=False)


def _moe_samples():
    import random

    rng = random.Random(3)
    out = []
    for i in range(4):
        P, R = rng.randint(4, 10), rng.randint(6, 20)
        out.append({"tokens": torch.tensor([rng.randrange(2048) for _ in range(P + R)]),
                    "mask_assistant": torch.tensor([0] * P + [1] * R),
                    "logprobs": torch.tensor([0.0] * P + [-2.0] * R), "advantage": torch.tensor([1.0 - 0.5 * i]),
                    "reward": torch.tensor([float(i % 2)]), "weight_version": torch.tensor([0])})
    return out


@pytest.mark.timeout(300)
def test_expert_parallel_trainer_step_matches_single_rank():
    """EP=2 x DP=2 PPO step (dense grads summed over DP, expert grads produced by the owner from every
    rank's dispatched tokens) equals one process on the whole batch (one mini-batch of 4 = 2 per rank):
    the dense gradient is identical on both ranks, each rank's expert gradient equals the matching slice."""
    ref = _moe_trainer(mini=4)
    samples = _moe_samples()
    ref.train_step(samples)
    want = {s.name: ref.flat.view(ref.flat.grad, s.name).clone() for s in ref.flat.slots}
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_trainer_worker, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=240) for _ in range(2))
    for p in ps:
        p.join(timeout=60)
    for rank in range(2):
        got = res[rank]
        assert not isinstance(got, str), got
        for name, w in got.items():
            w = torch.from_numpy(w)
            ref_w = want[name]
            if ".moe.w13" in name or ".moe.w2" in name:
                n = ref_w.shape[0] // 2
                ref_w = ref_w[rank * n:(rank + 1) * n]
            err = ((w - ref_w).norm() / ref_w.norm().clamp_min(1e-12)).item()
            assert err < 1e-4, (name, err)
