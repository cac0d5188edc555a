"""Context-parallel attention that reads every rank's K / V in place over NVLink (needs 2 GPUs; one process
per GPU).

The peer path (symmetric K / V buffers, device barriers, tcgen05 attention kernel with one TMA tensor map
per rank) must give the same output and the same dQ / dK / dV as the gathered path (NCCL all-gather of
K / V, chunked attention, reduce-scatter), and the output must match causal attention over the full rows
in fp32. Two calls in a row exercise the reuse of the symmetric buffers behind the barriers.
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


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


def _run_rank(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), LOCAL_WORLD_SIZE=str(world))
        torch.cuda.set_device(rank)
        from datetime import timedelta

        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                                timeout=timedelta(seconds=60))
        from meshy_b200.ops._ext import ext
        from meshy_b200.parallel.cp import CpLayout, CpSharder

        C = ext()
        C.clear_device_error()
        sh = CpSharder(dist.group.WORLD)
        rows, H, Hkv, hd = 2, 12, 2, 128
        for call, c in enumerate((256, 128)):
            S = 2 * world * c
            g = torch.Generator(device="cuda").manual_seed(10 + call)  # the same full rows on every rank
            full = [(torch.randn(rows, S, n, hd, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
                    for n in (H, Hkv, Hkv, H)]
            layout = CpLayout(rows, S, c)
            idx = sh.local_index(S, "cuda")
            local = [t[:, idx].reshape(rows * 2 * c, t.shape[2], hd).contiguous() for t in full]
            results = {}
            for mode in ("1", "0"):
                os.environ["MESHY_CP_PEER"] = mode
                qq, kk, vv = (t.clone().requires_grad_(True) for t in local[:3])
                assert sh.peer_ok(qq, layout) == (mode == "1")
                out = sh.attention(qq, kk, vv, layout)
                out.backward(local[3])
                torch.cuda.synchronize()
                results[mode] = (out.detach(), qq.grad, kk.grad, vv.grad)
            assert int(C.device_error()) == 0
            for a, b, name in zip(results["1"], results["0"], ("out", "dq", "dk", "dv")):
                r = _rel(a, b)
                assert r < 1e-2, (call, name, r)
            # the output against causal attention over the full rows (fp32)
            qf, kf, vf = (t.float().transpose(1, 2) for t in full[:3])
            kf = kf.repeat_interleave(H // Hkv, 1)
            vf = vf.repeat_interleave(H // Hkv, 1)
            ref = torch.nn.functional.scaled_dot_product_attention(qf, kf, vf, is_causal=True)
            ref = ref.transpose(1, 2)[:, idx].reshape(rows * 2 * c, H, hd)
            r = _rel(results["1"][0], ref)
            assert r < 2e-2, ("vs fp32", call, r)
        os.environ.pop("MESHY_CP_PEER", None)
        sh.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception:
        import traceback

        q.put((rank, traceback.format_exc()))


def test_cp_peer_attention_matches_gathered():
    if torch.cuda.device_count() < NEED:
        pytest.skip(f"needs {NEED} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_run_rank, args=(r, NEED, port, q)) for r in range(NEED)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=300)
    out = dict(q.get(timeout=5) for _ in range(NEED))
    for p in ps:
        if p.is_alive():
            p.kill()
    assert all(v == "ok" for v in out.values()), out
