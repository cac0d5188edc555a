"""Expert parallelism over NVLink peer memory (2 GPUs, one process per GPU, NCCL for set-up only).

Each rank routes its own tokens, the dispatch kernel stores the token rows straight into the experts'
owners, the owners run the grouped GEMMs on their local experts, and the return kernel stores the
outputs back. The result must equal the single-GPU native MoE layer applied to each rank's tokens, for
the output, the token gradient, the routing-weight gradient and each rank's slice of the expert weight
gradients, across two consecutive calls (the regions are reused).
"""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp_min(1e-12)).item()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _weights(E, D, F):
    g = torch.Generator(device="cuda").manual_seed(3)
    w13 = (torch.randn(E, 2 * F, D, device="cuda", generator=g) / D ** 0.5).to(torch.bfloat16)
    w2 = (torch.randn(E, D, F, device="cuda", generator=g) / F ** 0.5).to(torch.bfloat16)
    return w13, w2


def _inputs(rank, call, T, D, E, k):
    g = torch.Generator(device="cuda").manual_seed(100 * call + rank)
    x = torch.randn(T + 5 * rank, D, device="cuda", generator=g).to(torch.bfloat16)
    logits = torch.randn(x.shape[0], E, device="cuda", generator=g)
    p = torch.softmax(logits, -1)
    w, e = torch.topk(p, k, -1)
    w = w / w.sum(-1, keepdim=True)
    gout = torch.randn(x.shape[0], D, device="cuda", generator=g).to(torch.bfloat16)
    return x, w, e.int(), gout


def _worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), LOCAL_WORLD_SIZE=str(world))
        torch.cuda.set_device(rank)
        import torch.distributed as dist
        from datetime import timedelta

        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                                timeout=timedelta(seconds=120))
        from meshy_b200.ops import moe as M
        from meshy_b200.parallel.ep import PeerExchange, _PeerExperts

        E, D, F, k, T = 8, 256, 128, 2, 300
        w13, w2 = _weights(E, D, F)
        n = E // world
        w13_l = w13[rank * n:(rank + 1) * n].clone()
        w2_l = w2[rank * n:(rank + 1) * n].clone()
        xch = PeerExchange(dist.group.WORLD, D, (T + 5 * (world - 1)) * k, torch.device("cuda", rank))
        worst = {}
        for call in range(2):
            x, w, e, gout = _inputs(rank, call, T, D, E, k)
            x1 = x.clone().requires_grad_(True)
            w1 = w.clone().requires_grad_(True)
            w13_l.main_grad = torch.zeros(w13_l.shape, dtype=torch.float32, device="cuda")
            w2_l.main_grad = torch.zeros(w2_l.shape, dtype=torch.float32, device="cuda")
            out = _PeerExperts.apply(x1, w1, e, w13_l, w2_l, xch, 64)
            out.backward(gout)
            torch.cuda.synchronize()
            # reference: the full layer on this GPU, for this rank's tokens; the expert-weight gradient of
            # the EP layer sums every rank's tokens, so it is checked against the sum of both ranks' parts
            x2 = x.clone().requires_grad_(True)
            w2r = w.clone().requires_grad_(True)
            w13.main_grad = torch.zeros(w13.shape, dtype=torch.float32, device="cuda")
            w2.main_grad = torch.zeros(w2.shape, dtype=torch.float32, device="cuda")
            for r in range(world):
                xr, wr, er, gr = _inputs(r, call, T, D, E, k)
                xr.requires_grad_(True)  # the other ranks' tokens only feed the expert-weight gradients
                if r == rank:
                    xr, wr = x2, w2r
                ref = M.experts_forward(xr, wr, er, w13, w2, 64)
                ref.backward(gr)
                if r == rank:
                    ref_out = ref.detach()
            torch.cuda.synchronize()
            errs = {"out": _rel(out, ref_out), "dx": _rel(x1.grad, x2.grad), "dw": _rel(w1.grad, w2r.grad),
                    "dw13": _rel(w13_l.main_grad, w13.main_grad[rank * n:(rank + 1) * n]),
                    "dw2": _rel(w2_l.main_grad, w2.main_grad[rank * n:(rank + 1) * n])}
            for key, v in errs.items():
                worst[key] = max(worst.get(key, 0.0), v)
        import meshy_b200._C as C

        q.put((rank, worst, int(C.device_error())))
        dist.barrier()
        xch.close()
        dist.destroy_process_group()
    except Exception:
        import traceback

        q.put((rank, traceback.format_exc(), None))


@pytest.mark.timeout(300)
def test_expert_parallel_over_peer_memory_matches_local_layer():
    world = 2
    if torch.cuda.device_count() < world:
        pytest.skip("needs 2 GPUs")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = [q.get(timeout=240) for _ in range(world)]
    for p in ps:
        p.join(timeout=60)
    for rank, worst, err in res:
        assert not isinstance(worst, str), worst
        assert err == 0, (rank, err)
        assert worst["out"] < 1e-2 and worst["dx"] < 2e-2 and worst["dw"] < 2e-2, (rank, worst)
        assert worst["dw13"] < 2e-2 and worst["dw2"] < 2e-2, (rank, worst)
