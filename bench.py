"""Headline benchmark: JustRL lock-step GRPO step, per-GPU weak scaling.

Per rank (one process per GPU, ``torchrun`` for N > 1):
  R1-Distill-Qwen-1.5B architecture, bf16, random init; 8 prompts x group 8 =
  64 samples per GPU (64 prompts x 8 over 8 GPUs); prompt ids uniform random,
  length U[64, 512]; response lengths log-normal (median 2048, sigma 0.6, cap
  8192), generated to exactly that length (ignore EOS); binary rule reward
  (parity of the response id sum, p ~ 0.5); GRPO advantages; packed
  micro-batches; behaviour log-prob recompute; PPO mini-batches of 8 samples
  (the recipe's ``mini_batch_size``); DDP gradient all-reduce; AdamW; weight
  sync trainer -> rollout engine every step.

Timing: W untimed warm-up steps, then K timed steps bracketed by a barrier and
``torch.cuda.synchronize()``; CUDA events on the launching stream; max over
ranks.  Weights (3.6 GB) and KV pages far exceed the 126 MB L2, so no flush is
needed between steps.  SM clocks and throttle reasons are sampled with
nvidia-smi during the timed region.

``--impl reference`` runs the unmodified reference from ``baseline/_ref``
through its own public API, or prints why it cannot.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import random
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PHASES = ("rollout_s", "wait_s", "train_compute_s", "optim_s")
METRIC = "RL step time & trained tokens/s (JustRL 1.5B, 8 GPU); weight-sync latency"
BASELINE_VALUE = None  # the reference publishes no number for this metric


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=2)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="ours", choices=["ours", "reference", "torch"])
    p.add_argument("--prompts-per-gpu", type=int, default=8)
    p.add_argument("--group", type=int, default=8)
    p.add_argument("--median-resp", type=int, default=2048)
    p.add_argument("--resp-cap", type=int, default=8192)
    p.add_argument("--sigma", type=float, default=0.6)
    p.add_argument("--model", default="qwen2_5_math:R1-Distill-1.5B")
    p.add_argument("--max-tokens-per-micro", type=int, default=None,
                   help="packed micro-batch token budget (default 32768; 16384 for --impl torch, whose eager "
                        "autograd keeps every activation: 16384 is the reference recipe's seq_len with one "
                        "sample per micro)")
    p.add_argument("--no-clocks", action="store_true")
    return p.parse_args()


def reference_arm(args):
    """Run the unmodified reference (``baseline/_ref``) through its public API, or say exactly why not.

    The reference's headline run is ``scripts/launch.py --recipe recipe.justrl``: the Meshy control plane
    (``meshy.service.ignite``) drives SGLang inference servers (``sglang.launch_server``) and a torchtitan
    trainer through TransferQueue. Each module that path imports is tried in turn and the first errors are
    reported verbatim."""
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "meshy")):
        print(json.dumps({"impl": "reference", "unavailable": "baseline/_ref is not installed (no meshy package)"}))
        return
    sys.path.insert(0, ref)
    import importlib

    needed = ["meshy.config", "meshy.service.ignite", "meshy.engine.sglang", "meshy.backend.titan.trainer",
              "meshy.transferqueue", "sglang", "sglang.srt.entrypoints.http_server", "sgl_kernel",
              "transfer_queue", "tensordict"]
    errors = []
    for mod in needed:
        try:
            importlib.import_module(mod)
        except BaseException as e:  # noqa: BLE001 - report whatever the import raised
            errors.append(f"{mod}: {type(e).__name__}: {str(e).splitlines()[0] if str(e) else ''}"[:200])
    if errors:
        print(json.dumps({"impl": "reference", "unavailable": "import failed -- " + "; ".join(errors)}))
        return
    # not reached in this image: SGLang and TransferQueue are missing, so the recipe cannot start
    print(json.dumps({"impl": "reference", "unavailable": "every reference import succeeded, but the package install "
                      "does not ship the reference's scripts/launch.py that starts recipe.justrl"}))


class ClockSampler:
    def __init__(self, enabled: bool, index: int):
        self.enabled = enabled
        self.proc = None
        import tempfile

        self.path = os.path.join(tempfile.gettempdir(), f"meshy_bench_clocks_{os.getpid()}_rank{index}.csv")
        self.index = index

    def __enter__(self):
        if self.enabled:
            try:
                os.makedirs(os.path.dirname(self.path), exist_ok=True)
                self.f = open(self.path, "w")
                self.proc = subprocess.Popen(
                    ["nvidia-smi", "-i", str(self.index),
                     "--query-gpu=index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                     "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                     "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                     "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
            except Exception:
                self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self):
        if self.proc is None:
            return None
        try:
            rows = [l.strip().split(",") for l in open(self.path) if l.strip()]
        except Exception:
            return None
        sm = [float(r[1]) for r in rows if len(r) >= 9 and r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if len(r) >= 9 and r[2].strip().replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            if len(r) < 9:
                continue
            for name, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(sm)}


def make_workload(args, rank: int, step: int):
    rng = random.Random(1234 + 7919 * rank + 104729 * step)
    prompts = [[rng.randrange(151936) for _ in range(rng.randint(64, 512))] for _ in range(args.prompts_per_gpu)]
    mu = math.log(args.median_resp)
    lens = [max(1, min(args.resp_cap, int(round(math.exp(rng.gauss(mu, args.sigma))))))
            for _ in range(args.prompts_per_gpu * args.group)]
    return prompts, lens


def main():
    args = parse()
    if args.impl == "reference":
        reference_arm(args)
        return
    if args.max_tokens_per_micro is None:
        args.max_tokens_per_micro = 16384 if args.impl == "torch" else 32768
    # expandable segments for both arms: with the fixed-size segments the largest step (200k tokens) spent
    # 3.1 s in its training forward instead of ~0.8 s (the allocator reorganising its cache); expandable
    # segments brought it to 1.4 s
    os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = None
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=600))
        group = dist.group.WORLD

    from meshy_b200.config import TrainerConfig, TrainerParamsConfig
    from meshy_b200.ops import functional as Fx
    from meshy_b200.rl import ColocatedGRPO

    if args.impl == "torch":
        Fx.set_torch_baseline(True)
    name, flavor = args.model.split(":")
    max_len = 512 + args.resp_cap + 64
    tc = TrainerConfig(model_name=name, model_flavor=flavor, seq_len=max(8192, 1 << math.ceil(math.log2(max_len))),
                       lr=1e-6, weight_decay=0.1, max_norm=1.0, dtype="bfloat16", dp_replicate_degree=world,
                       steps=1000)
    tp = TrainerParamsConfig(mini_batch_size=8, batch_layout="packed", max_tokens_per_micro=args.max_tokens_per_micro,
                             ppo_clip_eps_low=0.2, ppo_clip_eps_high=0.28, old_logprobs_source="train",
                             log_entropy=True)
    rl = ColocatedGRPO(tc, tp, device=dev, group_size=args.group, dp_group=group, seed=0,
                       engine_kwargs=dict(max_running=args.prompts_per_gpu * args.group,
                                          # FlashAttention-2's paged decode (the baseline's) wants 256-token pages
                                          page_size=256 if args.impl == "torch" else 64,
                                          max_seq_len=max_len, mem_fraction=0.25, sync_every=16))
    try:
        C = __import__("meshy_b200._C", fromlist=["_C"])
    except Exception:
        C = None

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for w in range(args.warmup):
        prompts, lens = make_workload(args, rank, w)
        rl.step(prompts, lens)
    barrier()
    launches0 = C.launch_count() if (C is not None and hasattr(C, "launch_count")) else None
    graph0 = rl.engine.stats.get("graph_kernels", 0)
    tokens = 0
    resp_tokens = 0
    sync_ms = []
    phases = []
    times = []
    e2e_ms = []
    h2d = d2h = 0
    with ClockSampler(not args.no_clocks, local) as clocks:
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        barrier()
        start.record()
        for s in range(args.steps):
            prompts, lens = make_workload(args, rank, 100 + s)
            # end-to-end: prompts arrive as a pinned host tensor; the loss is read back
            flat = torch.tensor([t for p in prompts for t in p], dtype=torch.int64).pin_memory()
            h2d += flat.numel() * flat.element_size()
            t0 = time.perf_counter()
            dev_prompts = flat.to(dev, non_blocking=True)
            off = 0
            plist = []
            host = dev_prompts.cpu().tolist()
            for p in prompts:
                plist.append(host[off:off + len(p)])
                off += len(p)
            rep = rl.step(plist, lens)
            loss = torch.tensor([rep.metrics["pg_loss"]], device=dev).cpu()
            d2h += 4 + 8 * len(host)
            e2e_ms.append((time.perf_counter() - t0) * 1e3)
            if rank == 0:
                st = rl.engine.stats
                print(f"[bench] step {s}: rollout {rep.times['rollout_s']:.2f}s train {rep.times['train_s']:.2f}s "
                      f"sync {rep.times['weight_sync_ms']:.2f}ms tokens {rep.n_tokens} resp {rep.n_response_tokens} "
                      f"decode_steps {st['decode_steps']} "
                      + " ".join(f"{k}={v:.3f}" for k, v in rep.metrics.items() if k.startswith("time/")),
                      file=sys.stderr, flush=True)
            tokens += rep.n_tokens
            resp_tokens += rep.n_response_tokens
            sync_ms.append(rep.times["weight_sync_ms"])
            phases.append([rep.times.get(k, 0.0) for k in PHASES])
            del loss
        end.record()
        barrier()
    ms = start.elapsed_time(end)
    launches = None
    if launches0 is not None:
        launches = C.launch_count() - launches0 + (rl.engine.stats.get("graph_kernels", 0) - graph0)

    from meshy_b200.utils.timer import max_over_ranks

    # per-rank phase times of every timed step, gathered after the timed region: rollout (ends with the
    # host reading the generations), wait at the step's first collective, the rest of the train phase,
    # and the gradient reduction + optimiser buckets (CUDA-event device time)
    ph = torch.tensor(phases, dtype=torch.float64, device=dev)
    if world > 1:
        allph = [torch.empty_like(ph) for _ in range(world)]
        dist.all_gather(allph, ph)
        ph = torch.stack(allph)  # [rank, step, phase]
    else:
        ph = ph[None]
    phase_summary = {k: {"max_over_ranks_s": round(float(ph[:, :, i].max(0).values.mean()), 3),
                         "min_over_ranks_s": round(float(ph[:, :, i].min(0).values.mean()), 3)}
                     for i, k in enumerate(PHASES)}
    if rank == 0:
        for s_i in range(ph.shape[1]):
            print(f"[bench] phases step {s_i}: " + " ".join(
                f"{k}=[{float(ph[:, s_i, i].min()):.3f}..{float(ph[:, s_i, i].max()):.3f}]"
                for i, k in enumerate(PHASES)), file=sys.stderr, flush=True)

    ms_max = max_over_ranks(ms, group, dev)
    e2e_max = max_over_ranks(sum(e2e_ms), group, dev)
    sync_max = max_over_ranks(max(sync_ms), group, dev)
    tok_all = tokens
    if world > 1:
        t = torch.tensor([tokens, resp_tokens], dtype=torch.float64, device=dev)
        dist.all_reduce(t)
        tok_all, resp_tokens = int(t[0].item()), int(t[1].item())
    value = tok_all / (ms_max / 1e3)
    e2e_value = tok_all / (e2e_max / 1e3)
    n_params = rl.trainer.model_args.num_params()
    sync_bytes = rl.trainer.flat.numel * (2 + 2)  # read the bf16 compute weights, write the engine's copy
    meas = os.path.join(ROOT, "MEASURED_PEAKS.json")
    hbm = json.load(open(meas)).get("hbm_gbs", 6650.0) if os.path.exists(meas) else 6650.0
    if rank == 0:
        line = {
            "metric": METRIC,
            "value": round(value, 1),
            "unit": "trained tokens/s (all GPUs)",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_max / args.steps, 2),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None if BASELINE_VALUE is None else round(value / BASELINE_VALUE, 4),
            "dtype": "bf16",
            "data": "synthetic (random prompt ids, log-normal forced response lengths, random-init weights)",
            "impl": "torch-baseline" if args.impl == "torch" else "ours",
            "config": {
                "model": f"R1-Distill-Qwen-1.5B ({name}:{flavor}, {n_params / 1e9:.3f}B params)",
                "global_batch": args.prompts_per_gpu * args.group * world,
                "prompts_x_group": f"{args.prompts_per_gpu * world}x{args.group}",
                "seq_len": f"prompt U[64,512] + response lognormal(median {args.median_resp}, sigma {args.sigma}, "
                           f"cap {args.resp_cap})",
                "parallelism": f"dp{world} colocated (rollout TP1 per GPU)",
                "mini_batch_size": 8,
                "max_tokens_per_micro": args.max_tokens_per_micro,
                "l2": "inputs larger than L2 (3.6 GB bf16 weights per step)",
                "trained_tokens_per_step": tok_all // args.steps,
                "response_tokens_per_step": resp_tokens // args.steps,
            },
            "weight_sync": {"ms": round(sync_max, 3), "bytes": sync_bytes,
                            "roofline_ms": round(sync_bytes / (hbm * 1e9) * 1e3, 3),
                            "frac_of_measured_hbm": round((sync_bytes / (hbm * 1e9) * 1e3) / max(sync_max, 1e-9), 3),
                            "path": "trainer bf16 compute weights -> engine bf16 buffer, one device copy (colocated)"},
            "e2e": {"value": round(e2e_value, 1), "unit": "trained tokens/s (all GPUs)",
                    "h2d_bytes_per_step": h2d // args.steps, "d2h_bytes_per_step": d2h // args.steps},
            "gpu_launches": launches,
            "phases_per_step": phase_summary,
        }
        cs = clocks.summary()
        if cs is not None:
            line["clocks"] = cs
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
