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


class _EmulatedExchange:
    """One emulated rank's view of the exchange: its own regions, and address tables that list every emulated
    rank's regions (all on this GPU)."""

    def __init__(self, rank, world, dim, cap, regions, tables):
        self.rank, self.world, self.dim, self.cap = rank, world, dim, cap
        for name, bufs in regions.items():
            setattr(self, name, bufs[rank])
        for name, tab in tables.items():
            setattr(self, "t_" + name, tab)

    def owner_plan(self, experts, e_local):
        from meshy_b200.parallel.ep import PeerExchange

        return PeerExchange.owner_plan(self, experts, e_local)


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
@pytest.mark.parametrize("world", [2, 4])
def test_expert_parallel_kernels_emulated_on_one_gpu(world):
    """Every rank's phases run in turn on one GPU (dispatch for all, then the owners, then the sources): the
    dispatch / return kernels only store through address tables and never wait on another rank, so the
    exchange is exercised without a second GPU. Same oracle as the 2-GPU test."""
    from meshy_b200.ops import moe as M
    from meshy_b200.parallel import ep as EP

    E, D, F, k, T = 8, 256, 128, 2, 300
    w13, w2 = _weights(E, D, F)
    n_l = E // world
    cap = (T + 5 * (world - 1)) * k
    dev = "cuda"
    regions = {
        "recv_x": [torch.zeros(world * cap, D, dtype=torch.bfloat16, device=dev) for _ in range(world)],
        "recv_meta": [torch.zeros(world * cap, dtype=torch.int32, device=dev) for _ in range(world)],
        "recv_idx": [torch.zeros(world * cap, dtype=torch.int32, device=dev) for _ in range(world)],
        "recv_cnt": [torch.zeros(world, dtype=torch.int32, device=dev) for _ in range(world)],
        "ret": [torch.zeros(cap, D, dtype=torch.bfloat16, device=dev) for _ in range(world)],
    }
    tables = {name: torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device=dev)
              for name, bufs in regions.items()}
    xs = [_EmulatedExchange(r, world, D, cap, regions, tables) for r in range(world)]
    w13_l = [w13[r * n_l:(r + 1) * n_l].clone() for r in range(world)]
    w2_l = [w2[r * n_l:(r + 1) * n_l].clone() for r in range(world)]
    for r in range(world):
        w13_l[r].main_grad = torch.zeros(w13_l[r].shape, dtype=torch.float32, device=dev)
        w2_l[r].main_grad = torch.zeros(w2_l[r].shape, dtype=torch.float32, device=dev)
    inp = [_inputs(r, 0, T, D, E, k) for r in range(world)]
    # forward: sources, owners, sources
    disp = [EP._fwd_dispatch(inp[r][0], inp[r][2], xs[r], n_l) for r in range(world)]
    own = [EP._fwd_owner(xs[r], w13_l[r], w2_l[r]) for r in range(world)]
    col = [EP._fwd_collect(xs[r], inp[r][0].shape[0] * k, inp[r][1], inp[r][0].shape[0]) for r in range(world)]
    # backward
    dws = [EP._bwd_dispatch(inp[r][3], col[r][1], col[r][2], inp[r][1], *disp[r], n_l, xs[r]) for r in range(world)]
    for r in range(world):
        ids, slot, off, cnt, row_src, idx, xp, h, act = own[r]
        EP._bwd_owner(xs[r], ids, slot, off, row_src, idx, xp, h, act, w13_l[r], w2_l[r], 64)
    dxs = [EP._bwd_collect(xs[r], col[r][2], inp[r][0].shape[0]) for r in range(world)]
    torch.cuda.synchronize()
    # oracle: the local layer with every expert, rank by rank
    w13.main_grad = torch.zeros(w13.shape, dtype=torch.float32, device=dev)
    w2.main_grad = torch.zeros(w2.shape, dtype=torch.float32, device=dev)
    for r in range(world):
        x, w, e, gout = inp[r]
        x1, w1 = x.clone().requires_grad_(True), w.clone().requires_grad_(True)
        ref = M.experts_forward(x1, w1, e, w13, w2, 64)
        ref.backward(gout)
        assert _rel(col[r][0], ref) < 1e-2
        assert _rel(dxs[r], x1.grad) < 2e-2
        assert _rel(dws[r], w1.grad) < 2e-2
    for r in range(world):
        assert _rel(w13_l[r].main_grad, w13.main_grad[r * n_l:(r + 1) * n_l]) < 2e-2
        assert _rel(w2_l[r].main_grad, w2.main_grad[r * n_l:(r + 1) * n_l]) < 2e-2
