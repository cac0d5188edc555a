"""Context parallelism on CPU (gloo, 2 ranks): the head-tail sharded PPO step equals the unsharded one.

Each CP rank keeps chunks r and 2cp-1-r of every padded row, attention runs against the all-gathered
K/V with exact causal masking at global positions, dK/dV are reduce-scattered back, and gradients are
summed over the loss group: loss and gradient must match a single-process run."""

import os
import random
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _samples(seed=0, n=4):
    rng = random.Random(seed)
    out = []
    for i in range(n):
        P, R = rng.randint(4, 12), rng.randint(6, 30)
        toks = [rng.randrange(2048) for _ in range(P + R)]
        out.append({"tokens": torch.tensor(toks), "mask_assistant": torch.tensor([0] * P + [1] * R),
                    "logprobs": torch.tensor([0.0] * P + [-2.0] * R), "advantage": torch.tensor([1.0 - 0.5 * i]),
                    "reward": torch.tensor([float(i % 2)]), "weight_version": torch.tensor([0])})
    return out


def _trainer(cp_group=None, loss_group=None, old_source="train"):
    from meshy_b200.backend.trainer import PPOTrainer
    from meshy_b200.config import TrainerConfig, TrainerParamsConfig

    tc = TrainerConfig(model_name="qwen3", model_flavor="debugmodel", seq_len=64, lr=1e-3, weight_decay=0.0,
                       max_norm=0.0, dtype="float32", cp_degree=2 if cp_group is not None else 1)
    tp = TrainerParamsConfig(mini_batch_size=4, batch_layout="padded", micro_batch_size=2,
                             old_logprobs_source=old_source, seq_bucket=8)
    return PPOTrainer(tc, tp, device="cpu", seed=0, cp_group=cp_group, loss_group=loss_group, timer_enabled=False)


def _worker(rank, world, port, q, old_source="train"):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        g = dist.new_group([0, 1])
        t = _trainer(cp_group=g, loss_group=g, old_source=old_source)
        m = t.train_step(_samples())
        # by value: shared tensors die with the worker
        q.put((rank, t.flat.grad.numpy().copy(), m["pg_loss"], m["ess_ratio"]))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        import traceback

        q.put((rank, traceback.format_exc(), None, None))


@pytest.mark.timeout(300)
def test_context_parallel_step_matches_single_rank():
    ref = _trainer()
    m_ref = ref.train_step(_samples())
    want = ref.flat.grad.clone()  # the (single) mini-batch's gradient, reduced over the loss group
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=240) for _ in range(2)]
    for p in ps:
        p.join(timeout=60)
    for rank, got, loss, _ in res:
        assert not isinstance(got, str), got
        got = torch.from_numpy(got)
        assert abs(loss - m_ref["pg_loss"]) < 1e-4 * max(1.0, abs(m_ref["pg_loss"])), (loss, m_ref["pg_loss"])
        err = ((got - want).norm() / want.norm()).item()
        assert err < 1e-4, err


def _run_cp2(old_source):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q, old_source)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=240) for _ in range(2)]
    for p in ps:
        p.join(timeout=60)
    return res


@pytest.mark.timeout(300)
def test_effective_sample_size_is_cp_invariant():
    """Behaviour log-probs from the rollout make the importance ratios differ from 1, so the per-sequence
    effective sample size is non-trivial; split over two CP ranks it must equal the unsplit value (each
    sequence's ratio sums are combined over the CP group before the ESS is formed)."""
    ref = _trainer(old_source="rollout")
    want = ref.train_step(_samples())["ess_ratio"]
    assert 0.0 < want < 1.0
    for rank, grad, loss, ess in _run_cp2("rollout"):
        assert not isinstance(grad, str), grad
        assert abs(ess - want) < 1e-5, (rank, ess, want)


def test_head_tail_shard_and_gather_indices():
    from meshy_b200.parallel.cp import CpSharder

    class _S(CpSharder):
        def __init__(self, size, rank):
            self.size, self.rank, self.group = size, rank, None

    S = 16
    parts = [_S(2, r).local_index(S).tolist() for r in range(2)]
    assert parts == [[0, 1, 2, 3, 12, 13, 14, 15], [4, 5, 6, 7, 8, 9, 10, 11]]
    order = _S(2, 0).gather_order(S)
    cat = torch.tensor(parts[0] + parts[1])
    assert cat[order].tolist() == list(range(S))
