"""Rollout-only benchmark: prefill + paged-KV decode throughput of the rollout engine.

Counterpart of the train-only benchmark (reference ``scripts/bench_train_only.py``
times the trainer without inference); this one times the inference half of the
RL step without the trainer.  Random-init weights of the named architecture,
``--batch`` prompts of ``--prompt-len`` random ids, each forced to decode
``--gen`` tokens (EOS ignored).  Decode is timed with CUDA events around whole
engine steps (each step = ``--sync-every`` graph replays + one host sync).

    python -m meshy_b200.bench.rollout --batch 64 --prompt-len 2048 --gen 256

Prints one JSON line: prefill tokens/s, decode ms per step, decode tokens/s,
and the weight + KV bytes one decode step must read (for the HBM roofline).
"""

from __future__ import annotations

import argparse
import json
import os
import random
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--model", default="qwen2_5_math:R1-Distill-1.5B")
    p.add_argument("--batch", type=int, default=64)
    p.add_argument("--prompt-len", type=int, default=512)
    p.add_argument("--gen", type=int, default=256)
    p.add_argument("--sync-every", type=int, default=16)
    p.add_argument("--no-graph", action="store_true")
    p.add_argument("--torch-baseline", action="store_true", help="cuBLAS/torch path (comparison only)")
    args = p.parse_args(argv)

    import torch

    from meshy_b200.models import get_model_args
    from meshy_b200.ops import functional as Fx
    from meshy_b200.rollout import RolloutEngine

    if args.torch_baseline:
        Fx.set_torch_baseline(True)
    name, flavor = args.model.split(":")
    margs = get_model_args(name, flavor)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    max_len = args.prompt_len + args.gen + 64
    eng = RolloutEngine(margs, device=dev, max_running=args.batch, page_size=64, max_seq_len=max_len,
                        max_total_tokens=args.batch * (max_len + 2 * args.sync_every + 64),
                        use_cuda_graph=not args.no_graph, sync_every=args.sync_every, seed=0,
                        prefill_chunk_tokens=args.batch * args.prompt_len)
    rng = random.Random(0)
    prompts = [[rng.randrange(margs.vocab_size) for _ in range(args.prompt_len)] for _ in range(args.batch)]

    # warm-up round: captures the graphs for this batch bucket
    eng.generate(prompts[: max(1, args.batch)], 2 * args.sync_every, ignore_eos=True)
    torch.cuda.synchronize()

    for pr in prompts:
        eng.submit(pr, args.gen, ignore_eos=True)
    t0, t1, t2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    t0.record()
    while eng.waiting:
        eng._admit()  # prefill of the whole batch (one packed forward)
    t1.record()
    torch.cuda.synchronize()
    steps0 = eng.stats["decode_steps"]
    tok0 = eng.stats["decode_tokens"]
    w0 = time.perf_counter()
    while eng.has_work():
        eng.step()
    t2.record()
    torch.cuda.synchronize()
    wall_decode_ms = (time.perf_counter() - w0) * 1e3
    eng.finished.clear()
    prefill_ms = t0.elapsed_time(t1)
    decode_ms = t1.elapsed_time(t2)
    steps = eng.stats["decode_steps"] - steps0
    dtoks = eng.stats["decode_tokens"] - tok0
    w_bytes = eng.weight_flat.numel() * eng.weight_flat.element_size()
    avg_ctx = args.prompt_len + args.gen / 2
    kv_bytes = args.batch * avg_ctx * margs.kv_bytes_per_token(2)
    step_ms = decode_ms / max(1, steps)
    meas = os.path.join(ROOT, "MEASURED_PEAKS.json")
    hbm = json.load(open(meas)).get("hbm_gbs", 6650.0) if os.path.exists(meas) else 6650.0
    roof_ms = (w_bytes + kv_bytes) / (hbm * 1e9) * 1e3
    print(json.dumps({
        "bench": "rollout", "model": args.model, "batch": args.batch, "prompt_len": args.prompt_len, "gen": args.gen,
        "impl": "torch-baseline" if args.torch_baseline else "ours", "cuda_graph": not args.no_graph,
        "decode_path": "whole-step kernel" if eng._mega is not None and args.batch <= 64 else
        f"per-op kernels ({eng.mega_reason or 'batch > 64'})",
        "prefill_ms": round(prefill_ms, 2), "prefill_tok_s": round(args.batch * args.prompt_len / prefill_ms * 1e3),
        "decode_steps": steps, "decode_ms_per_step": round(step_ms, 4),
        "decode_wall_ms_per_step": round(wall_decode_ms / max(1, steps), 4),
        "decode_tok_s": round(dtoks / decode_ms * 1e3), "bytes_per_step": int(w_bytes + kv_bytes),
        "roofline_ms_per_step": round(roof_ms, 4), "frac_of_measured_hbm": round(roof_ms / step_ms, 3),
    }), flush=True)


if __name__ == "__main__":
    main()
