"""Fused data-parallel optimiser step (``csrc/kernels/symm.cu``) on one GPU: HBM roofline of its kernels.

The step is a barrier, the reduce-scatter with the shard's sum of squares, the norm exchange, the AdamW update
with the bf16 push, and a closing barrier. With one rank the address tables hold only this GPU's buffers, so
no NVLink traffic is involved and the kernels can be timed (CUDA events) and profiled by themselves; the
multi-GPU step adds (world - 1) x 4 bytes of peer reads and (world - 1) x 2 bytes of peer stores per shard
element.

    python -m meshy_b200.bench.dp_step --numel 268435456

Bytes per element of the shard (one rank, sharded fp32 master): reduce-scatter 4 read + 4 written; AdamW
16 read (master, gradient, two moments) + 12 written (master, two moments) + 2 (bf16 push).
"""

from __future__ import annotations

import argparse
import json

import torch


def main() -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--numel", type=int, default=1 << 28)
    p.add_argument("--iters", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    args = p.parse_args()
    from ..ops._ext import ext
    from .ops import peaks

    C = ext()
    dev = torch.device("cuda", torch.cuda.current_device())
    n = args.numel // 4 * 4
    f32 = torch.float32
    grad = torch.randn(n, device=dev) * 1e-3
    local_grad = torch.empty(n, dtype=f32, device=dev)
    master = torch.randn(n, device=dev) * 0.02
    compute = torch.empty(n, dtype=torch.bfloat16, device=dev)
    m = torch.zeros(n, dtype=f32, device=dev)
    v = torch.zeros(n, dtype=f32, device=dev)
    flags = torch.zeros(1, dtype=torch.int32, device=dev)
    slots = torch.zeros(1, dtype=f32, device=dev)
    scalars = torch.zeros(2, dtype=f32, device=dev)

    def tab(t):
        return torch.tensor([t.data_ptr()], dtype=torch.int64, device=dev)

    t_grad, t_compute, t_flags, t_slots = tab(grad), tab(compute), tab(flags), tab(slots)
    epoch = 0

    def step(i):
        nonlocal epoch
        epoch += 3
        C.symm_dp_adamw(t_grad, None, t_compute, t_flags, t_slots, master, local_grad, m, v, scalars, 0, 1, 0, n,
                        epoch, 1.0, 1e-5, 0.9, 0.999, 1e-8, 0.01, i + 1, 10.0)

    # the step touches 38 bytes per element (10 GB at the default size), far more than the 126 MB L2, so
    # back-to-back steps need no flush between them
    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(args.iters):
        step(args.warmup + i)
    b.record()
    b.synchronize()
    if int(C.device_error()):
        raise SystemExit(f"device error {int(C.device_error())}")
    ms = a.elapsed_time(b) / args.iters
    bytes_moved = n * (8 + 30)
    hbm, _, src = peaks()
    out = {"op": "fused_dp_step_world1", "numel": n, "ms": round(ms, 4), "gb": round(bytes_moved / 1e9, 3),
           "gbs": round(bytes_moved / ms / 1e6, 1), "frac_of_hbm": round(bytes_moved / ms / 1e6 / hbm, 3),
           "peak_source": src}
    print(json.dumps(out))


if __name__ == "__main__":
    main()
