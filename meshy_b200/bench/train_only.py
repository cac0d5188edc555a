"""Training-only benchmark (reference ``scripts/bench_train_only.py``): no inference engine, no data plane.

Every rank builds the same :class:`~meshy_b200.backend.trainer.PPOTrainer`
(any DP / CP / TP / EP layout of the replica), takes the first ``N`` rows of a
``trajectories.jsonl`` written with ``verbose_trajectory_log=True`` (token
ids, masks, log-probs) -- or synthetic rows of the given length distribution
when no file is given -- plans the batch and times ``--steps`` train steps
over it with CUDA events (max over ranks).  Prints one JSON line: step time,
trained tokens/s, model TFLOP/s (6 N tokens), peak memory and plan stats.

    python -m meshy_b200.bench.train_only --num-samples 64 --steps 3
    torchrun --nproc-per-node 8 -m meshy_b200.bench.train_only --cp 2 --layout padded \\
        --model qwen3:8B --seq-len 16384 --num-samples 128
    ... --plan legacy   # the pre-dynamic-batching baseline: fixed [micro_batch_size, seq_len] blocks
"""

from __future__ import annotations

import argparse
import json
import math
import os
import random
import statistics
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def read_records(path: str, n: int) -> list[dict]:
    out = []
    with open(path, encoding="utf-8") as fh:
        for line in fh:
            line = line.strip()
            if not line:
                continue
            r = json.loads(line)
            if "tokens" not in r:
                raise ValueError(f"{path}: rows need token ids (write the log with verbose_trajectory_log=True)")
            out.append(r)
            if len(out) >= n:
                break
    return out


def synthetic_records(n: int, vocab: int, median: int, sigma: float, cap: int, seed: int = 0) -> list[dict]:
    rng = random.Random(seed)
    out = []
    for i in range(n):
        P = rng.randint(64, 512)
        R = max(1, min(cap, int(round(math.exp(rng.gauss(math.log(median), sigma))))))
        out.append({"tokens": [rng.randrange(vocab) for _ in range(P + R)], "masks": [0] * P + [1] * R,
                    "logprobs": [0.0] * P + [-1.0] * R, "reward": float(i % 2), "advantage": 1.0 - 2.0 * (i % 2)})
    return out


def to_samples(records):
    import torch

    out = []
    for r in records:
        m = r.get("mask_assistant", r.get("masks"))
        out.append({"tokens": torch.tensor(r["tokens"]), "mask_assistant": torch.tensor(m),
                    "logprobs": torch.tensor(r.get("logprobs", [0.0] * len(r["tokens"])), dtype=torch.float32),
                    "advantage": torch.tensor([float(r.get("advantage", 0.0))]),
                    "reward": torch.tensor([float(r.get("reward", 0.0))]),
                    "weight_version": torch.tensor([int(r.get("weight_version", 0))])})
    return out


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--model", default="qwen2_5_math:R1-Distill-1.5B")
    p.add_argument("--trajectories", default=None)
    p.add_argument("--num-samples", type=int, default=64)
    p.add_argument("--steps", type=int, default=3)
    p.add_argument("--warmup", type=int, default=1)
    p.add_argument("--seq-len", type=int, default=16384)
    p.add_argument("--layout", choices=["packed", "padded"], default="packed")
    p.add_argument("--max-tokens-per-micro", type=int, default=32768)
    p.add_argument("--micro-batch-size", type=int, default=1)
    p.add_argument("--mini-batch-size", type=int, default=8)
    p.add_argument("--plan", choices=["dynamic", "legacy"], default="dynamic")
    p.add_argument("--cp", type=int, default=1)
    p.add_argument("--tp", type=int, default=1)
    p.add_argument("--ep", type=int, default=1)
    p.add_argument("--median-resp", type=int, default=2048)
    p.add_argument("--sigma", type=float, default=0.6)
    p.add_argument("--resp-cap", type=int, default=8192)
    p.add_argument("--old-logprobs", choices=["train", "rollout"], default="train")
    p.add_argument("--json-out", default=None)
    args = p.parse_args(argv)

    import torch
    import torch.distributed as dist

    from meshy_b200.config import TrainerConfig, TrainerParamsConfig
    from meshy_b200.engine.trainer import TrainerEngine
    from meshy_b200.models import get_model_args
    from meshy_b200.utils.timer import max_over_ranks

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    cuda = torch.cuda.is_available()
    dev = torch.device("cuda", local) if cuda else torch.device("cpu")
    if cuda:
        torch.cuda.set_device(dev)
    name, flavor = args.model.split(":")
    margs = get_model_args(name, flavor)
    tc = TrainerConfig(model_name=name, model_flavor=flavor, seq_len=args.seq_len, lr=1e-6, weight_decay=0.1,
                       max_norm=1.0, dtype="bfloat16" if cuda else "float32", cp_degree=args.cp, tp_degree=args.tp,
                       ep_degree=args.ep)
    legacy = args.plan == "legacy"
    tp = TrainerParamsConfig(mini_batch_size=args.mini_batch_size,
                             batch_layout="padded" if legacy else args.layout,
                             max_tokens_per_micro=None if (legacy or args.layout == "padded") else
                             args.max_tokens_per_micro,
                             micro_batch_size=args.micro_batch_size, old_logprobs_source=args.old_logprobs)
    eng = TrainerEngine(tc, tp, service_name="bench", rank=rank, world_size=world,
                        master_addr=os.environ.get("MASTER_ADDR", "127.0.0.1"),
                        master_port=int(os.environ.get("MASTER_PORT", "29500")), device=dev)
    if world > 1 and not dist.is_initialized():
        eng.init_process_group()
    eng.setup()
    t = eng.trainer
    rec = read_records(args.trajectories, args.num_samples) if args.trajectories else synthetic_records(
        args.num_samples, margs.vocab_size, args.median_resp, args.sigma, args.resp_cap)
    samples = to_samples(rec)
    plan = t.plan_batch(samples, t.dp_size)
    local_s = plan.local_samples(samples, t.dp_rank)
    tokens = sum(min(len(s["tokens"]), args.seq_len) for s in samples)
    for _ in range(args.warmup):
        t.train_step(local_s, plan=plan.per_rank[t.dp_rank])
    if cuda:
        torch.cuda.synchronize()
        torch.cuda.reset_peak_memory_stats(dev)
    times = []
    for _ in range(args.steps):
        if world > 1:
            dist.barrier()
        if cuda:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            a.record()
        import time

        w0 = time.perf_counter()
        t.train_step(local_s, plan=plan.per_rank[t.dp_rank])
        if cuda:
            b.record()
            torch.cuda.synchronize()
            ms = a.elapsed_time(b)
        else:
            ms = (time.perf_counter() - w0) * 1e3
        times.append(max_over_ranks(ms, t.loss_group if world > 1 else None, dev))
    step_ms = statistics.median(times)
    peak = torch.cuda.max_memory_allocated(dev) / 2**30 if cuda else 0.0
    n_params = margs.num_params()
    stats = {k: float(v) for k, v in __import__("meshy_b200.backend.plan", fromlist=["plan_stats"]).plan_stats(
        plan.per_rank[t.dp_rank], t.batch_layout).items()}
    out = {"bench": "train_only", "model": args.model, "n_gpus": world, "samples": len(samples), "tokens": tokens,
           "layout": t.batch_layout, "plan": args.plan, "cp": args.cp, "tp": args.tp, "ep": args.ep,
           "step_ms": round(step_ms, 2), "tokens_per_s": round(tokens / (step_ms / 1e3), 1),
           "model_tflops": round(6 * n_params * tokens / (step_ms / 1e3) / 1e12, 1),
           "old_logprobs_recompute": args.old_logprobs == "train", "peak_mem_gib": round(peak, 2),
           "plan_stats": stats}
    if rank == 0:
        print(json.dumps(out), flush=True)
        if args.json_out:
            with open(args.json_out, "w") as f:
                json.dump(out, f, indent=1)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
