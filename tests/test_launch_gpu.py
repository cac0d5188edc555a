"""The launcher product path on a GPU: launcher → bootstrap store + column store → ignitor → native engine
server colocated with the trainer in a FALLBACK / ON_DEMAND ring → rollout driver, through three weight
versions with the device weight sync (CUDA IPC snapshots, no disk export between steps).

Mirrors the reference's integration smoke (``scripts/smoke/run.sh:87-179``: the run must advance the
weight version every step). ``MESHY_LAUNCH_GPU_CARDS`` (default 1) sets the card count; more cards than
the box has skip the test.
"""

import json
import os
import re
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.timeout(900)
def test_launcher_colocated_grpo_with_device_weight_sync(tmp_path):
    cards = int(os.environ.get("MESHY_LAUNCH_GPU_CARDS", "1"))
    if torch.cuda.device_count() < cards:
        pytest.skip(f"needs {cards} GPUs")
    env = dict(os.environ, XRL_DEVICE="cuda", XRL_SMOKE_STEPS="3", XRL_SMOKE_CARDS=str(cards),
               XRL_SMOKE_WEIGHT_SYNC="device", PYTHONPATH=ROOT, NCCL_NVLS_ENABLE="0",
               XRL_PORT_OFFSET=str(100 + (_free_port() % 400) * 10))
    rt = tmp_path / "rt"
    proc = subprocess.Popen([sys.executable, "-m", "meshy_b200.launch", "--recipe", "recipe.justrl_smoke",
                             "--runtime-dir", str(rt), "--master-port", str(_free_port())], cwd=ROOT, env=env,
                            stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True, start_new_session=True)
    timed_out = False
    try:
        out, _ = proc.communicate(timeout=int(os.environ.get("MESHY_LAUNCH_GPU_TIMEOUT", "600")))
    except subprocess.TimeoutExpired:
        timed_out = True
        import signal

        os.killpg(proc.pid, signal.SIGTERM)
        out, _ = proc.communicate(timeout=60)
    logs = rt / "logs"
    detail = (out or "")[-3000:]
    if logs.exists():
        for f in sorted(logs.iterdir()):
            detail += f"\n==== {f.name}\n" + f.read_text(errors="replace")[-2500:]
    if timed_out or proc.returncode != 0:
        print(detail)
    assert not timed_out, "launcher run timed out\n" + detail
    assert proc.returncode == 0, detail
    rows = [json.loads(l) for l in (rt / "tensorboard" / "actor_train-0" / "metrics.jsonl").read_text().splitlines()]
    assert len(rows) == 3, detail
    # every engine loaded versions 1..3 from the trainer snapshot on its own GPU, with no disk export
    syncs = []
    for f in sorted(logs.iterdir()):
        syncs += re.findall(r"\[weight-sync\] ipc version (\d+) local=(\w+) ([0-9.]+) ms", f.read_text(errors="replace"))
    versions = sorted(int(v) for v, _, _ in syncs)
    assert versions == sorted(list(range(1, 4)) * cards), (syncs, detail)
    assert all(loc == "True" for _, loc, _ in syncs), syncs
    assert not (rt / "weights").exists() or not any((rt / "weights").rglob("*.safetensors")), detail
    ms = [float(x) for _, _, x in syncs]
    print(f"device weight sync over {cards} card(s): {len(ms)} loads, max {max(ms):.2f} ms")
