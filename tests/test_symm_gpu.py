"""Fused DP optimiser step over NVLink peer memory (needs 2 GPUs; one process per GPU).

* numerics: reduce-scatter + global norm + clip + AdamW + all-gather by P2P stores gives the same master /
  compute weights as "NCCL all-reduce of the gradient + the fp32 AdamW definition" on every rank;
* failure detection without a GPU fault: one rank never arrives at the device barrier; the other rank's
  bounded wait gives up after 1 s, records the error code, and the context stays usable.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

NEED = 2


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), LOCAL_WORLD_SIZE=str(world))
    torch.cuda.set_device(rank)
    from datetime import timedelta

    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=timedelta(seconds=60))


def _numerics(rank, world, port, q):
    try:
        _init(rank, world, port)
        from meshy_b200.backend.flat import FlatParams
        from meshy_b200.models import build_model, get_model_args
        from meshy_b200.ops.reference import adamw_
        from meshy_b200.parallel.symm import FusedDPAdamW

        args = get_model_args("qwen3", "debugmodel")
        model = build_model(args, seed=0, device="cuda", dtype=torch.float32)
        flat = FlatParams(model, compute_dtype=torch.bfloat16, device="cuda")
        g = torch.Generator(device="cuda").manual_seed(100 + rank)
        flat.grad.copy_(torch.randn(flat.numel, device="cuda", generator=g) * 1e-2)
        # reference: all-reduce + clip + AdamW on copies
        ref_p = flat.master.clone()
        ref_g = flat.grad.clone()
        dist.all_reduce(ref_g)
        norm = float(ref_g.norm())
        scale = min(1.0, 0.5 / (norm + 1e-6))
        m, v = torch.zeros_like(ref_p), torch.zeros_like(ref_p)
        adamw_(ref_p, ref_g, m, v, lr=1e-3, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1, step=1,
               grad_scale=scale)
        opt = FusedDPAdamW(flat, None, lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, max_norm=0.5,
                           timeout_s=20.0)
        gn = opt.step()
        torch.cuda.synchronize()
        opt.check()
        # the fp32 master is sharded like the moments (only bf16 is replicated by the step): gather it to compare
        flat.gather_master()
        assert abs(float(gn) - norm) <= 1e-4 * norm, (float(gn), norm)
        err = (flat.master - ref_p).abs().max().item()
        assert err < 1e-6, err
        assert torch.equal(flat.compute, flat.master.to(torch.bfloat16))
        # every rank holds the same weights
        other = flat.master.clone()
        dist.broadcast(other, 0)
        assert torch.equal(other, flat.master)
        # ZeRO-1 moments: each rank keeps its shard; the gathered moments equal the reference's
        assert flat.exp_avg.numel() == opt.hi - opt.lo
        fm, fv = opt.full_moments()
        assert (fm - m).abs().max().item() <= 1e-6 * max(1.0, m.abs().max().item())
        assert (fv - v).abs().max().item() <= 1e-5 * v.abs().max().item()
        opt.heap.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:  # report to the parent
        import traceback

        q.put((rank, traceback.format_exc()))


def _timeout(rank, world, port, q):
    try:
        _init(rank, world, port)
        from meshy_b200.ops._ext import ext
        from meshy_b200.parallel.symm import SymmetricHeap

        heap = SymmetricHeap(4096)
        _, flags = heap.alloc(world, torch.int32)
        dist.barrier()
        C = ext()
        C.clear_device_error()
        if rank == 0:
            C.symm_barrier(flags, 0, world, 1000, 1.0)  # rank 1 never arrives at epoch 1000
            torch.cuda.synchronize()
            code = int(C.device_error())
            C.clear_device_error()
            torch.cuda.synchronize()
            x = torch.ones(4, device="cuda") * 2  # the context is still usable
            assert float(x.sum()) == 8.0
            q.put((rank, f"code={code}"))
        else:
            q.put((rank, "skipped"))
        dist.barrier()
        heap.close()
        dist.destroy_process_group()
    except Exception:
        import traceback

        q.put((rank, traceback.format_exc()))


def _run(fn):
    if torch.cuda.device_count() < NEED:
        pytest.skip(f"needs {NEED} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=fn, args=(r, NEED, port, q)) for r in range(NEED)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=300)
    out = dict(q.get(timeout=5) for _ in range(NEED))
    for p in ps:
        if p.is_alive():
            p.kill()
    return out


def test_fused_dp_adamw_matches_allreduce_reference():
    out = _run(_numerics)
    assert all(v == "ok" for v in out.values()), out


def test_symm_barrier_times_out_with_error_code():
    out = _run(_timeout)
    assert out[0] == "code=4", out
