"""Per-op benchmark of the hot kernels at the flagship model's shapes.

Times each op with CUDA events on the launching stream after warm-up. Between
timed launches a 256 MiB buffer is read (not written, so L2 holds no dirty
lines that the timed op would have to write back), so every launch starts with
a cold L2 (126 MB). Reports the median time, the bytes or FLOPs the op must move
or compute, and the fraction of the measured HBM copy bandwidth or cuBLAS bf16
throughput (``MEASURED_PEAKS.json``; the pool's earlier measurement if absent).

    python -m meshy_b200.bench.ops --suite decode --batch 64
    python -m meshy_b200.bench.ops --suite train --tokens 16384

Prints one JSON line per op.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        d = json.load(open(path))
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), "measured"
    return 6650.0, 1590.0, "fallback"


def time_op(fn, iters=20, warmup=5):
    import torch

    flush = torch.ones(64 << 20, dtype=torch.float32, device="cuda")
    sink = torch.empty((), dtype=torch.float32, device="cuda")
    for _ in range(warmup):
        fn()
    times = []
    for _ in range(iters):
        torch.sum(flush, dim=0, out=sink)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b) * 1e3)
    times.sort()
    return times[len(times) // 2]


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--suite", choices=["decode", "train"], default="decode")
    p.add_argument("--model", default="qwen2_5_math:R1-Distill-1.5B")
    p.add_argument("--batch", type=int, nargs="*", default=[8, 64, 256])
    p.add_argument("--ctx", type=int, default=2048, help="decode context length per sequence")
    p.add_argument("--tokens", type=int, default=16384, help="tokens per micro-batch (train suite)")
    p.add_argument("--torch-baseline", action="store_true", help="time cuBLAS (torch.matmul) for the GEMMs")
    p.add_argument("--cluster", type=int, default=0, help="small-M GEMM cluster split-K size (0 = heuristic)")
    p.add_argument("--no-small-m", action="store_true", help="decode GEMMs through the regular 128-row tiling")
    p.add_argument("--ops", default="", help="comma-separated subset of ops to run")
    args = p.parse_args(argv)

    import torch

    import meshy_b200._C as C
    from meshy_b200.models import get_model_args

    hbm, tflops, src = peaks()
    C.gemm_small_config(0 if args.no_small_m else 1, args.cluster)
    only = set(filter(None, args.ops.split(",")))
    name, flavor = args.model.split(":")
    a = get_model_args(name, flavor)
    D, F, V, hd = a.dim, a.ffn_dim, a.vocab_size, a.head_dim
    qkv_n = (a.n_heads + 2 * a.n_kv_heads) * hd
    dev = "cuda"
    torch.manual_seed(0)
    lin = {
        "qkv": (qkv_n, D), "o": (D, a.n_heads * hd), "gate_up": (2 * F, D), "down": (D, F), "lm_head": (V, D),
    }
    W = {k: (torch.randn(n, kk, device=dev) * 0.02).to(torch.bfloat16) for k, (n, kk) in lin.items()}

    def emit(rec):
        rec.update(peak_source=src, cluster=args.cluster, small_m=not args.no_small_m)
        print(json.dumps(rec), flush=True)

    if args.suite == "decode":
        for M in args.batch:
            for k, w in W.items():
                if only and k not in only:
                    continue
                n, kk = w.shape
                x = torch.randn(M, kk, device=dev).to(torch.bfloat16)
                out = torch.empty(M, n, device=dev, dtype=torch.bfloat16)
                if args.torch_baseline:
                    fn = lambda: torch.matmul(x, w.t(), out=out)  # noqa: E731
                elif k == "gate_up":
                    out = torch.empty(M, n // 2, device=dev, dtype=torch.bfloat16)
                    fn = lambda: C.gemm(x, w, out, False, False, None, None, None, 1, False, 64)  # noqa: E731
                else:
                    fn = lambda: C.gemm(x, w, out, False, False, None, None, None, 0, False, 0)  # noqa: E731
                us = time_op(fn)
                byts = w.numel() * 2 + x.numel() * 2 + out.numel() * 2
                emit(dict(op=f"gemm_{k}", M=M, N=n, K=kk, us=round(us, 2), bytes=byts,
                          gbs=round(byts / us / 1e3, 1), frac_of_hbm=round(byts / us / 1e3 / hbm, 3),
                          impl="cublas" if args.torch_baseline else "ours"))
            if not only or "lm_sample" in only:
                # LM head + sampler: the regular 128-row tiling vs the small-M path (M <= 64)
                n, kk = W["lm_head"].shape
                h = torch.randn(M, kk, device=dev).to(torch.bfloat16)
                tok = torch.empty(M, dtype=torch.int64, device=dev)
                lp = torch.empty(M, device=dev)
                step = torch.zeros(1, dtype=torch.int64, device=dev)
                byts = W["lm_head"].numel() * 2
                impls = [("regular", lambda: C.lmhead_sample(h, W["lm_head"], tok, lp, 1.0, 0, step))]
                if M <= 64:
                    impls.append(("small_m", lambda: C.lmhead_sample_small(h, W["lm_head"], None, 0, 0.0, 0.0, tok,
                                                                           lp, 1.0, 0, step)))
                for impl, fn in impls:
                    us = time_op(fn)
                    emit(dict(op="lm_sample", M=M, N=n, K=kk, us=round(us, 2), bytes=byts,
                              gbs=round(byts / us / 1e3, 1), frac_of_hbm=round(byts / us / 1e3 / hbm, 3), impl=impl))
            if only and "paged_decode" not in only:
                continue
            # paged decode attention
            page = 64
            pages_per = (args.ctx + page - 1) // page
            n_pages = M * pages_per + 1
            kc = torch.randn(n_pages, a.n_kv_heads, page, hd, device=dev).to(torch.bfloat16)
            vc = torch.randn_like(kc)
            bt = torch.arange(1, n_pages, device=dev, dtype=torch.int32).view(M, pages_per)
            seq = torch.full((M,), args.ctx, device=dev, dtype=torch.int32)
            q = torch.randn(M, a.n_heads, hd, device=dev).to(torch.bfloat16)
            o = torch.empty_like(q)
            ws = torch.empty(M * a.n_heads * 64 * (hd + 2), device=dev)
            us = time_op(lambda: C.paged_attention(q, kc, vc, bt, seq, o, 1 / math.sqrt(hd), ws))
            byts = 2 * M * args.ctx * a.n_kv_heads * hd * 2
            emit(dict(op="paged_decode", B=M, ctx=args.ctx, us=round(us, 2), bytes=byts,
                      gbs=round(byts / us / 1e3, 1), frac_of_hbm=round(byts / us / 1e3 / hbm, 3)))
    else:
        T = args.tokens
        for k, w in W.items():
            if only and k not in only:
                continue
            n, kk = w.shape
            x = torch.randn(T, kk, device=dev).to(torch.bfloat16)
            out = torch.empty(T, n, device=dev, dtype=torch.bfloat16)
            if args.torch_baseline:
                fn = lambda: torch.matmul(x, w.t(), out=out)  # noqa: E731
            else:
                fn = lambda: C.gemm(x, w, out, False, False, None, None, None, 0, False, 0)  # noqa: E731
            us = time_op(fn, iters=10)
            fl = 2.0 * T * n * kk
            emit(dict(op=f"gemm_{k}", M=T, N=n, K=kk, us=round(us, 2), tflops=round(fl / us / 1e6, 1),
                      frac_of_bf16=round(fl / us / 1e6 / tflops, 3), impl="cublas" if args.torch_baseline else "ours"))
        if only and "flash_attn" not in only:
            return
        # packed causal attention, forward and backward (MESHY_FA_TC=0: the mma.sync kernels)
        hq, hkv, hd = a.n_heads, a.n_kv_heads, a.head_dim
        for lens in ([2048] * 8, [4096] * 4, [1300] * 8, [16384]):
            Tt = sum(lens)
            q = torch.randn(Tt, hq, hd, device=dev).to(torch.bfloat16)
            kx = torch.randn(Tt, hkv, hd, device=dev).to(torch.bfloat16)
            vx = torch.randn(Tt, hkv, hd, device=dev).to(torch.bfloat16)
            cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32, device=dev)
            o = torch.empty_like(q)
            lse = torch.empty(hq, Tt, device=dev)
            sc = 1 / math.sqrt(hd)
            us_f = time_op(lambda: C.flash_attn_fwd(q, kx, vx, cu, o, lse, max(lens), sc), iters=10)
            go = torch.randn_like(q)
            gq, gk, gv = torch.empty_like(q), torch.empty_like(kx), torch.empty_like(vx)
            us_b = time_op(lambda: C.flash_attn_bwd(q, kx, vx, cu, o, go, lse, gq, gk, gv, max(lens), sc), iters=10)
            fl = sum(2.0 * L * L * hq * hd for L in lens)
            emit(dict(op="flash_attn", docs=f"{len(lens)}x{lens[0]}", fwd_us=round(us_f, 1),
                      fwd_tflops=round(fl / us_f / 1e6, 1), bwd_us=round(us_b, 1),
                      bwd_tflops=round(2.5 * fl / us_b / 1e6, 1),
                      impl="mma.sync" if os.environ.get("MESHY_FA_TC", "1") == "0" else "tcgen05"))


if __name__ == "__main__":
    main()
