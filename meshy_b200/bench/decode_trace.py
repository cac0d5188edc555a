"""Per-CTA timeline of the small-M GEMMs inside one replayed decode step (global-timer ns, no profiler).

Every small-M GEMM launch of the captured step writes, per CTA, eight global-timer stamps (``_C.gemm_small_trace``):
entry, producer past the dependency wait, first stage landed at the MMA, last MMA committed, accumulator ready
at the epilogue, partials exchanged (first cluster barrier), epilogue done, exit. The report gives, per GEMM of a
layer (QKV, o_proj, gate/up, down; means over the layers), the median CTA's phase lengths and the gap from the
previous traced launch's last exit to this launch's dependency release (for o_proj that gap holds the paged
attention kernel). The paged-attention launches are traced the same way (``_C.paged_decode_trace``): entry,
past the dependency wait, Q staged, first page consumed, last page consumed, CTA merge, cluster merge, exit.

    python -m meshy_b200.bench.decode_trace --batch 1 --prompt-len 2048
"""

from __future__ import annotations

import argparse
import json

import torch

PHASES = ("launch_to_wait", "wait_to_first_stage", "first_stage_to_last_mma", "last_mma_to_acc",
          "acc_to_exchanged", "exchanged_to_epilogue_done", "epilogue_to_exit")
KINDS = ("qkv", "o_proj", "gate_up", "down")


def main() -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--model", default="qwen2_5_math:R1-Distill-1.5B")
    p.add_argument("--batch", type=int, default=1)
    p.add_argument("--prompt-len", type=int, default=2048)
    p.add_argument("--gen", type=int, default=64)
    args = p.parse_args()
    from ..models import get_model_args
    from ..ops._ext import ext
    from ..rollout.engine import RolloutEngine

    name, flavor = args.model.split(":")
    margs = get_model_args(name, flavor)
    C = ext()
    L = margs.n_layers
    per_step = 4 * L + 1
    slots = 4 * per_step + 64
    buf = torch.zeros(slots, 160, 8, dtype=torch.int64, device="cuda")
    eng = RolloutEngine(margs, device="cuda", max_running=max(8, args.batch), max_seq_len=args.prompt_len + args.gen + 64,
                        seed=0)
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, margs.vocab_size, (args.prompt_len,), generator=g).tolist()
               for _ in range(args.batch)]
    # every small-M launch takes the next slot: the prefill's sampler, the capture's two warm-up runs, then the
    # captured step, whose slots every replay rewrites (all rows end together, so nothing launches after it)
    abuf = torch.zeros(4 * L + 16, 1024, 8, dtype=torch.int64, device="cuda")
    C.gemm_small_trace(buf)
    C.paged_decode_trace(abuf)
    eng.generate(prompts, args.gen, temperature=1.0, ignore_eos=True)
    torch.cuda.synchronize()
    C.gemm_small_trace(None)
    C.paged_decode_trace(None)
    t = buf.cpu()
    ta = abuf.cpu()
    used = [i for i in range(slots) if int(t[i, 0, 0]) != 0]
    step = used[-per_step:] if len(used) >= per_step else used
    rows = {k: {ph: [] for ph in PHASES + ("gap_from_prev_exit", "ctas")} for k in KINDS}
    prev_exit = None
    for j, s in enumerate(step):
        ctas = t[s][t[s, :, 0] != 0].double()
        if ctas.numel() == 0:
            continue
        kind = KINDS[j % 4] if j < 4 * L else "lm_head"
        med = ctas.median(0).values
        d = [float(med[i + 1] - med[i]) / 1e3 for i in range(7)]
        if kind in rows:
            for ph, v in zip(PHASES, d):
                rows[kind][ph].append(v)
            rows[kind]["ctas"].append(float(ctas.shape[0]))
            if prev_exit is not None:
                rows[kind]["gap_from_prev_exit"].append(float(ctas[:, 1].min() - prev_exit) / 1e3)
        prev_exit = float(ctas[:, 7].max())
    out = {"batch": args.batch, "prompt_len": args.prompt_len, "unit": "us (median CTA; mean over layers)"}
    for k in KINDS:
        out[k] = {ph: round(sum(v) / len(v), 2) for ph, v in rows[k].items() if v}
    ent = min(float(t[s][t[s, :, 0] != 0][:, 0].min()) for s in step)
    ext_ = max(float(t[s][t[s, :, 0] != 0][:, 7].max()) for s in step)
    out["traced_span_ms"] = round((ext_ - ent) / 1e6, 4)
    # decode attention: the captured step's launches are the last L used slots
    aused = [i for i in range(ta.shape[0]) if int(ta[i, 0, 0]) != 0][-L:]
    names = ("wait", "q_staged", "first_page", "other_pages", "cta_merge", "cluster_merge", "exit")
    acc = {n: [] for n in names + ("total_max_cta", "ctas")}
    for s_ in aused:
        ctas = ta[s_][ta[s_, :, 0] != 0].double()
        med = ctas.median(0).values
        for i, n in enumerate(names):
            acc[n].append(float(med[i + 1] - med[i]) / 1e3)
        acc["total_max_cta"].append(float(ctas[:, 7].max() - ctas[:, 0].min()) / 1e3)
        acc["ctas"].append(float(ctas.shape[0]))
    out["attention"] = {n: round(sum(v) / len(v), 2) for n, v in acc.items() if v}
    print(json.dumps(out, indent=1))


if __name__ == "__main__":
    main()
