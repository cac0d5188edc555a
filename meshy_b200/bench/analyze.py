"""Run-log analysis (reference ``scripts/analyze_step_timing.py``, ``scripts/analyze_trajectory_rewards.py``).

    python -m meshy_b200.bench.analyze step-timing  <runtime dir>
    python -m meshy_b200.bench.analyze rewards      <runtime dir> [--csv out.csv]

``step-timing`` splits the run's wall time per trainer step into rollout
(the card owned by the inference side), train, and hand-off, from the
colocation transfer lines of ``logs/ignitor-0.log`` and the trainer's
``tensorboard/<trainer>/metrics.jsonl`` (``perf/*``, ``time/train/*``).
``rewards`` reports, per weight version of ``trajectories.jsonl``: sample count,
mean reward, pass rate, mean response length, truncation rate, and the wall
clock between consecutive versions.  Only the few top-level fields needed are
read, so very large logs stream.
"""

from __future__ import annotations

import argparse
import csv
import glob
import json
import os
import re
import sys
from collections import defaultdict
from datetime import datetime

_TRANSFER = re.compile(r"^(\S+ \S+) .*colocation transfer (\S+) -> (\S+) \(seq=(\d+), (\S+)\)")


def _ts(s: str) -> float:
    return datetime.strptime(s, "%Y-%m-%d %H:%M:%S,%f").timestamp()


def step_timing(root: str) -> list[dict]:
    log = os.path.join(root, "logs", "ignitor-0.log")
    events = []
    if os.path.exists(log):
        for line in open(log, errors="replace"):
            m = _TRANSFER.match(line)
            if m:
                events.append((_ts(m.group(1)), m.group(2), m.group(3), int(m.group(4))))
    for f in glob.glob(os.path.join(root, "logs", "*-0.log")):
        for line in open(f, errors="replace"):
            m = _TRANSFER.match(line)
            if m:
                events.append((_ts(m.group(1)), m.group(2), m.group(3), int(m.group(4))))
    events = sorted(set(events), key=lambda e: (e[3], e[0]))
    metrics = []
    for f in glob.glob(os.path.join(root, "tensorboard", "*", "metrics.jsonl")):
        metrics += [json.loads(l) for l in open(f) if l.strip()]
    rows = []
    prev_to_infer = events[0][0] if events else None
    for i, (t, src, dst, seq) in enumerate(events):
        if dst == "actor_infer" or "infer" in dst:
            prev_to_infer = t
            continue
        nxt = next((e for e in events[i + 1:] if "infer" in e[2]), None)
        rows.append({"seq": seq, "owner": dst, "rollout_s": round(t - prev_to_infer, 3) if prev_to_infer else None,
                     "train_s": round(nxt[0] - t, 3) if nxt else None})
    for r, m in zip([r for r in rows if r["owner"] != "critic"], sorted(metrics, key=lambda x: x.get("step", 0))):
        r["step"] = m.get("step")
        for k in ("perf/step_time", "time/train/old_logprobs", "time/train/forward", "time/train/backward",
                  "time/train/optim_step"):
            if k in m:
                r[k] = round(float(m[k]), 4)
    return rows


def rewards(root: str) -> list[dict]:
    path = root if root.endswith(".jsonl") else os.path.join(root, "trajectories.jsonl")
    agg = defaultdict(lambda: {"n": 0, "reward": 0.0, "passed": 0, "tokens": 0, "truncated": 0, "t0": None})
    for line in open(path, errors="replace"):
        if not line.strip():
            continue
        r = json.loads(line)
        a = agg[int(r.get("weight_version", 0))]
        a["n"] += 1
        rew = float(r.get("raw_reward") if r.get("raw_reward") is not None else r.get("reward", 0.0))
        a["reward"] += float(r.get("reward", 0.0))
        a["passed"] += rew > 0.5
        a["tokens"] += int(r.get("n_tokens", 0))
        a["truncated"] += bool(r.get("truncated"))
        ts = r.get("timestamp")
        if ts is not None:
            a["t0"] = ts if a["t0"] is None else min(a["t0"], ts)
    out, prev = [], None
    for v in sorted(agg):
        a = agg[v]
        n = max(1, a["n"])
        row = {"weight_version": v, "samples": a["n"], "reward_mean": round(a["reward"] / n, 4),
               "pass_rate": round(a["passed"] / n, 4), "tokens_mean": round(a["tokens"] / n, 1),
               "truncated_rate": round(a["truncated"] / n, 4)}
        if a["t0"] is not None and prev is not None:
            row["wall_s_since_prev"] = round(a["t0"] - prev, 2)
        prev = a["t0"] if a["t0"] is not None else prev
        out.append(row)
    return out


def main(argv=None) -> int:
    p = argparse.ArgumentParser()
    sub = p.add_subparsers(dest="cmd", required=True)
    a = sub.add_parser("step-timing")
    a.add_argument("root")
    b = sub.add_parser("rewards")
    b.add_argument("root")
    b.add_argument("--csv", default=None)
    args = p.parse_args(argv)
    rows = step_timing(args.root) if args.cmd == "step-timing" else rewards(args.root)
    if getattr(args, "csv", None) and rows:
        with open(args.csv, "w", newline="") as f:
            w = csv.DictWriter(f, fieldnames=sorted({k for r in rows for k in r}))
            w.writeheader()
            w.writerows(rows)
    for r in rows:
        print(json.dumps(r))
    return 0


if __name__ == "__main__":
    sys.exit(main())
