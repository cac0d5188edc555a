"""Context-parallel attention benchmark: peer path (K/V read in place over NVLink) vs gathered path (NCCL
all-gather of K/V + chunked attention), one process per GPU.

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 -m meshy_b200.bench.cp_attention --seq 32768

Random bf16 q/k/v of ``--rows`` rows of ``--seq`` tokens (head-tail sharded over the ranks; 12 query heads,
2 KV heads, head_dim 128 as R1-Distill-1.5B). Times the forward alone (no grad) and forward + backward of
one attention layer with CUDA events after warm-up, takes the max over ranks, and prints one JSON line.
"""

from __future__ import annotations

import argparse
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--rows", type=int, default=1)
    p.add_argument("--seq", type=int, default=32768)
    p.add_argument("--iters", type=int, default=10)
    args = p.parse_args(argv)

    import torch
    import torch.distributed as dist

    from meshy_b200.parallel.cp import CpLayout, CpSharder

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    world, rank = dist.get_world_size(), dist.get_rank()
    sh = CpSharder(dist.group.WORLD)
    rows, S, H, Hkv, hd = args.rows, args.seq, 12, 2, 128
    c = S // (2 * world)
    layout = CpLayout(rows, S, c)
    n = rows * 2 * c
    g = torch.Generator(device="cuda").manual_seed(rank)
    q, k, v, go = ((torch.randn(n, h, hd, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
                   for h in (H, Hkv, Hkv, H))

    def timed(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.iters):
            fn()
        b.record()
        torch.cuda.synchronize()
        t = torch.tensor([a.elapsed_time(b) / args.iters], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t)

    res = {}
    for mode in ("peer", "gathered"):
        os.environ["MESHY_CP_PEER"] = "1" if mode == "peer" else "0"

        def fwd():
            with torch.no_grad():
                sh.attention(q, k, v, layout)

        def fwd_bwd():
            qq, kk, vv = (t.detach().requires_grad_(True) for t in (q, k, v))
            sh.attention(qq, kk, vv, layout).backward(go)

        res[mode] = {"fwd_ms": round(timed(fwd), 3), "fwd_bwd_ms": round(timed(fwd_bwd), 3)}
    # causal attention FLOPs of this rank's queries (4 * keys visible * hd per query head), forward
    fl = 0.0
    for chunk in sh.chunk_ids():
        start = chunk * c
        fl += rows * H * 4 * hd * (c * start + c * (c + 1) / 2)
    for mode in res:
        res[mode]["fwd_tflops_per_gpu"] = round(fl / (res[mode]["fwd_ms"] * 1e-3) / 1e12, 1)
    if rank == 0:
        print(json.dumps(dict(bench="cp_attention", world=world, rows=rows, seq=S, heads=H, kv_heads=Hkv,
                              head_dim=hd, timing="CUDA events, max over ranks", **res)), flush=True)
    sh.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
