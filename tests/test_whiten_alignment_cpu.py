"""Advantage whitening across data- and context-parallel ranks (CPU, gloo, 4 ranks = DP 2 x CP 2).

Before CP sharding every CP rank holds its DP slice's full sequences, so whitening must count each token once:
either reduce over the batch group (one rank per DP index) or over the whole DP x CP group with the CP degree
divided out. Both must give the single-process whitening of all unique tokens: ``(a - mean) / sqrt(var +
1e-8)`` with the unbiased variance, zero outside the mask.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from meshy_b200.backend.gae import whiten

SLICES = {0: [1.0, 2.0, 99.0], 1: [4.0, 8.0, 99.0]}  # the last token of each row is outside the mask
MASK = torch.tensor([[1.0, 1.0, 0.0]])


def _expected(dp):
    allv = torch.tensor([1.0, 2.0, 4.0, 8.0], dtype=torch.float64)
    z = (allv - allv.mean()) / torch.sqrt(allv.var() + 1e-8)
    return z[:2] if dp == 0 else z[2:]


def test_single_process_formula():
    a = torch.tensor([[2.0, 4.0, 1000.0]])
    out = whiten(a, MASK)
    assert torch.allclose(out, torch.tensor([[-2 ** -0.5, 2 ** -0.5, 0.0]]), atol=1e-6)
    assert whiten(torch.tensor([[2.0, 2.0, 5.0]]), MASK).abs().sum() == 0


def _worker(rank, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=4)
        from meshy_b200.parallel.mesh import build_parallel_dims

        pd = build_parallel_dims(4, rank, dp_replicate=-1, dp_shard=1, cp=2)
        adv = torch.tensor([SLICES[pd.dp_rank]])
        by_batch = whiten(adv, MASK, pd.batch_group)
        by_loss = whiten(adv, MASK, pd.loss_group, cp_degree=2)
        q.put((rank, pd.dp_rank, by_batch.numpy().copy(), by_loss.numpy().copy()))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        import traceback

        q.put((rank, traceback.format_exc(), None, None))


@pytest.mark.timeout(300)
def test_dp_by_cp_whitening_counts_each_token_once():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(4)]
    for p in ps:
        p.start()
    res = [q.get(timeout=240) for _ in range(4)]
    for p in ps:
        p.join(timeout=60)
    for rank, dp, by_batch, by_loss in res:
        assert not isinstance(dp, str), dp
        want = _expected(dp)
        for got in (by_batch, by_loss):
            got = torch.from_numpy(got)[0]
            assert torch.allclose(got[:2].double(), want, atol=1e-6), (rank, got)
            assert got[2] == 0
