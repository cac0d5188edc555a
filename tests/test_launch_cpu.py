"""End to end on CPU: launcher → bootstrap store + column store → torchrun ignitors (2 cards) →
inference servers colocated in a FALLBACK/ON_DEMAND ring with a DDP2 trainer (gloo) → rollout driver.

Mirrors the reference's integration smoke (``scripts/smoke/run.sh``: the run must advance the weight
version for N steps and write its artifacts) without a GPU.
"""

import json
import os
import socket
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _port_offset() -> str:
    """Shift every service port of this run so launcher tests running side by side do not collide."""
    return str(100 + (_free_port() % 400) * 10)


@pytest.mark.timeout(600)
def test_launcher_runs_colocated_grpo_on_cpu(tmp_path):
    env = dict(os.environ, XRL_DEVICE="cpu", XRL_SMOKE_STEPS="3", XRL_SMOKE_CKPT="1", PYTHONPATH=ROOT, XRL_PORT_OFFSET=_port_offset())
    port = _free_port()
    rt = tmp_path / "rt"
    r = subprocess.run([sys.executable, "-m", "meshy_b200.launch", "--recipe", "recipe.justrl_smoke",
                        "--runtime-dir", str(rt), "--master-port", str(port)], cwd=ROOT, env=env,
                       capture_output=True, text=True, timeout=540)
    logs = rt / "logs"
    detail = r.stdout[-2000:] + r.stderr[-2000:]
    if logs.exists():
        for f in sorted(logs.iterdir()):
            detail += f"\n==== {f.name}\n" + f.read_text(errors="replace")[-1500:]
    assert r.returncode == 0, detail
    # three trainer steps were logged, and the weight version advanced through the ring
    rows = [json.loads(l) for l in (rt / "tensorboard" / "actor_train-0" / "metrics.jsonl").read_text().splitlines()]
    assert len(rows) == 3, detail
    ev = [f for f in os.listdir(rt / "tensorboard" / "actor_train-0") if f.startswith("events.out.tfevents")]
    assert ev
    ign = (logs / "ignitor-0.log").read_text()
    assert ign.count("colocation transfer actor_infer -> actor_train") == 3, detail
    # trajectories and global checkpoints (trainer + rollout shards) exist
    assert (rt / "trajectories.jsonl").exists()
    state = rt / "state"
    assert (state / "actor_train-0").exists() and (state / "rollout-0").exists(), detail


@pytest.mark.timeout(600)
@pytest.mark.parametrize("moe", [False, True], ids=["dense-tp2", "moe-tp2-ep2"])
def test_launcher_runs_tensor_parallel_inference_replica_on_cpu(tmp_path, moe):
    """The ring with ONE inference replica over both cards (``--tp-size 2``: the service starts the server,
    which spawns its follower rank): the replica serves the rollout, releases and restores its memory in
    lock-step, loads every weight version and the run finishes. With the MoE model the replica's ranks also
    split the experts (``--ep-size 2``) and each loads only its experts' slices of every weight version."""
    env = dict(os.environ, XRL_DEVICE="cpu", XRL_SMOKE_STEPS="2", XRL_SMOKE_INFER_TP="2", PYTHONPATH=ROOT,
               XRL_PORT_OFFSET=_port_offset())
    if moe:
        env.update(XRL_SMOKE_MODEL="qwen3:debugmodel_moe", XRL_SMOKE_INFER_EP="2")
    rt = tmp_path / "rt"
    r = subprocess.run([sys.executable, "-m", "meshy_b200.launch", "--recipe", "recipe.justrl_smoke",
                        "--runtime-dir", str(rt), "--master-port", str(_free_port())], cwd=ROOT, env=env,
                       capture_output=True, text=True, timeout=540)
    logs = rt / "logs"
    detail = r.stdout[-2000:] + r.stderr[-2000:]
    if logs.exists():
        for f in sorted(logs.iterdir()):
            detail += f"\n==== {f.name}\n" + f.read_text(errors="replace")[-1500:]
    assert r.returncode == 0, detail
    rows = [json.loads(l) for l in (rt / "tensorboard" / "actor_train-0" / "metrics.jsonl").read_text().splitlines()]
    assert len(rows) == 2, detail
    assert (logs / "actor_infer-0-0.log").exists() and not (logs / "actor_infer-1-0.log").exists(), detail
    assert (logs / "ignitor-0.log").read_text().count("colocation transfer actor_infer -> actor_train") == 2, detail


@pytest.mark.timeout(600)
def test_two_node_launch_with_an_inference_replica_across_the_nodes(tmp_path):
    """Two launchers (``--nnodes 2``, one card each, on this host) run one job: the data plane and bootstrap
    store live on node 0, the trainer spans both nodes, and the single inference replica spans them too
    (node 0's server serves HTTP and rendezvouses with node 1's follower through ``--dist-init-addr``)."""
    env = dict(os.environ, XRL_DEVICE="cpu", XRL_SMOKE_STEPS="2", XRL_SMOKE_INFER_TP="2", PYTHONPATH=ROOT,
               XRL_PORT_OFFSET=_port_offset())
    rt = tmp_path / "rt"
    port = str(_free_port())
    procs = [subprocess.Popen([sys.executable, "-m", "meshy_b200.launch", "--recipe", "recipe.justrl_smoke",
                               "--runtime-dir", str(rt), "--nnodes", "2", "--node-rank", str(n),
                               "--nproc-per-node", "1", "--master-port", port], cwd=ROOT, env=env,
                              stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True) for n in (0, 1)]
    outs = [p.communicate(timeout=540)[0] for p in procs]
    logs = rt / "logs"
    detail = "".join(o[-1500:] for o in outs)
    if logs.exists():
        for f in sorted(logs.iterdir()):
            detail += f"\n==== {f.name}\n" + f.read_text(errors="replace")[-1500:]
    assert [p.returncode for p in procs] == [0, 0], detail
    rows = [json.loads(l) for l in (rt / "tensorboard" / "actor_train-0" / "metrics.jsonl").read_text().splitlines()]
    assert len(rows) == 2, detail
    # one server per node for the one replica
    assert (logs / "actor_infer-0-0.log").exists() and (logs / "actor_infer-0-1.log").exists(), detail
    assert (logs / "ignitor-0.log").read_text().count("colocation transfer actor_infer -> actor_train") == 2, detail


@pytest.mark.timeout(600)
@pytest.mark.parametrize("mode", ["bounded-off-policy", "fully-async-stream"])
def test_launcher_pacing_modes_on_cpu(tmp_path, mode):
    """The two non-lock-step pacing modes end to end. Bounded off-policy (colocated, ``pacing_window=2``):
    the rollout runs one window ahead, so the first two batches are generated with version 0 and the third
    with version 1. Fully asynchronous (disaggregated cards, no gate, ``stream_minibatch``): the trainer takes
    each 2-sample mini-batch as it arrives, syncing weights once per 8-sample batch."""
    env = dict(os.environ, XRL_DEVICE="cpu", XRL_SMOKE_STEPS="3", PYTHONPATH=ROOT, XRL_PORT_OFFSET=_port_offset())
    if mode == "bounded-off-policy":
        env.update(XRL_SMOKE_PACING="2")
    else:
        env.update(XRL_SMOKE_TOPOLOGY="disaggregate", XRL_SMOKE_PACING="none", XRL_SMOKE_STREAM="1")
    rt = tmp_path / "rt"
    r = subprocess.run([sys.executable, "-m", "meshy_b200.launch", "--recipe", "recipe.justrl_smoke",
                        "--runtime-dir", str(rt), "--master-port", str(_free_port())], cwd=ROOT, env=env,
                       capture_output=True, text=True, timeout=540)
    logs = rt / "logs"
    detail = r.stdout[-2000:] + r.stderr[-2000:]
    if logs.exists():
        for f in sorted(logs.iterdir()):
            detail += f"\n==== {f.name}\n" + f.read_text(errors="replace")[-1500:]
    assert r.returncode == 0, detail
    rows = [json.loads(l) for l in (rt / "tensorboard" / "actor_train-0" / "metrics.jsonl").read_text().splitlines()]
    versions = [json.loads(l)["weight_version"] for l in (rt / "trajectories.jsonl").read_text().splitlines()]
    assert len(versions) == 24, detail
    if mode == "bounded-off-policy":
        assert len(rows) == 3 and sorted(versions) == [0] * 16 + [1] * 8, (versions, detail)
    else:
        assert len(rows) == 12 and rows[-1]["step"] == 3, ([r_.get("step") for r_ in rows], detail)
        assert max(versions) <= 2  # generated ahead of the trainer, never ahead of its weights


@pytest.mark.timeout(600)
def test_launcher_runs_sharded_trainer_on_cpu(tmp_path):
    """The same ring with the trainer's parameters sharded over its two ranks (FSDP): weights still reach
    the engines every step (gathered into the full layout) and the run checkpoints and finishes."""
    env = dict(os.environ, XRL_DEVICE="cpu", XRL_SMOKE_STEPS="2", XRL_SMOKE_CKPT="1", XRL_SMOKE_SHARD="1",
               PYTHONPATH=ROOT, XRL_PORT_OFFSET=_port_offset())
    port = _free_port()
    rt = tmp_path / "rt"
    r = subprocess.run([sys.executable, "-m", "meshy_b200.launch", "--recipe", "recipe.justrl_smoke",
                        "--runtime-dir", str(rt), "--master-port", str(port)], cwd=ROOT, env=env,
                       capture_output=True, text=True, timeout=540)
    logs = rt / "logs"
    detail = r.stdout[-2000:] + r.stderr[-2000:]
    if logs.exists():
        for f in sorted(logs.iterdir()):
            detail += f"\n==== {f.name}\n" + f.read_text(errors="replace")[-1500:]
    assert r.returncode == 0, detail
    rows = [json.loads(l) for l in (rt / "tensorboard" / "actor_train-0" / "metrics.jsonl").read_text().splitlines()]
    assert len(rows) == 2, detail
    ign = (logs / "ignitor-0.log").read_text()
    assert ign.count("colocation transfer actor_infer -> actor_train") == 2, detail
    assert (rt / "state" / "actor_train-0").exists(), detail


@pytest.mark.timeout(600)
def test_launcher_runs_critic_ppo_on_cpu(tmp_path):
    """Ring of inference → critic → trainer on one card: the critic cold-starts for one window (it raises
    the gate itself), then publishes values that the trainer turns into VAPO-GAE advantages."""
    env = dict(os.environ, XRL_DEVICE="cpu", XRL_SMOKE_STEPS="2", XRL_SMOKE_COLD="1", PYTHONPATH=ROOT, XRL_PORT_OFFSET=_port_offset())
    rt = tmp_path / "rt"
    r = subprocess.run([sys.executable, "-m", "meshy_b200.launch", "--recipe", "recipe.justrl_ii_smoke",
                        "--runtime-dir", str(rt), "--master-port", str(_free_port())], cwd=ROOT, env=env,
                       capture_output=True, text=True, timeout=540)
    logs = rt / "logs"
    detail = r.stderr[-2000:]
    if logs.exists():
        for f in sorted(logs.iterdir()):
            detail += f"\n==== {f.name}\n" + f.read_text(errors="replace")[-1500:]
    assert r.returncode == 0, detail
    critic_log = (logs / "critic-0-0.log").read_text()
    assert "critic cold start 1" in critic_log and "critic window 3" in critic_log, detail
    rows = [json.loads(l) for l in (rt / "tensorboard" / "actor_train-0" / "metrics.jsonl").read_text().splitlines()]
    assert len(rows) == 2 and all("critic/value_mean" in x for x in rows), detail


@pytest.mark.timeout(600)
def test_launcher_runs_topk_distillation_on_cpu(tmp_path):
    """Inference → teacher (Top-K columns appended in place) → student trainer (forward KL over the teacher's
    Top-K), all ring members of one card."""
    env = dict(os.environ, XRL_DEVICE="cpu", XRL_SMOKE_STEPS="2", PYTHONPATH=ROOT, XRL_PORT_OFFSET=_port_offset())
    rt = tmp_path / "rt"
    r = subprocess.run([sys.executable, "-m", "meshy_b200.launch", "--recipe", "recipe.student_topk_opd_smoke",
                        "--runtime-dir", str(rt), "--master-port", str(_free_port())], cwd=ROOT, env=env,
                       capture_output=True, text=True, timeout=540)
    detail = r.stderr[-2000:]
    logs = rt / "logs"
    if logs.exists():
        for f in sorted(logs.iterdir()):
            detail += f"\n==== {f.name}\n" + f.read_text(errors="replace")[-1500:]
    assert r.returncode == 0, detail
    rows = [json.loads(l) for l in (rt / "tensorboard" / "actor_train-0" / "metrics.jsonl").read_text().splitlines()]
    assert len(rows) == 2 and all("train/distill_loss" in x and x["train/teacher_topk_mass"] > 0 for x in rows), detail


def _launch(rt, steps, *extra):
    env = dict(os.environ, XRL_DEVICE="cpu", XRL_SMOKE_STEPS=str(steps), XRL_SMOKE_CKPT="1", PYTHONPATH=ROOT, XRL_PORT_OFFSET=_port_offset())
    return subprocess.run([sys.executable, "-m", "meshy_b200.launch", "--recipe", "recipe.justrl_smoke",
                           "--runtime-dir", str(rt), "--master-port", str(_free_port()), *extra], cwd=ROOT, env=env,
                          capture_output=True, text=True, timeout=540)


@pytest.mark.timeout(900)
def test_kill_and_resume_on_cpu(tmp_path):
    """A run that stopped after two steps resumes from the newest step every participant committed: shards
    newer than that are dropped, the step counter continues from there, and reusing the directory without
    ``--resume`` is refused."""
    rt = tmp_path / "rt"
    r = _launch(rt, 2)
    assert r.returncode == 0, r.stderr[-3000:]
    state = rt / "state"
    trainer_done = sorted(int(f.split("-")[1].split(".")[0]) for f in os.listdir(state / "actor_train-0")
                          if f.endswith(".complete"))
    rollout_done = sorted(int(f.split("-")[1].split(".")[0]) for f in os.listdir(state / "rollout-0")
                          if f.endswith(".complete"))
    resume_at = max(set(trainer_done) & set(rollout_done))
    # a fresh start over a directory with checkpoints is an error
    r = _launch(rt, 3)
    text = r.stdout + r.stderr + "".join(f.read_text(errors="replace") for f in (rt / "logs").glob("ignitor-*.log"))
    assert r.returncode != 0 and "--resume was not passed" in text, text[-3000:]
    r = _launch(rt, 3, "--resume")
    ign = (rt / "logs" / "ignitor-0.log").read_text()
    assert r.returncode == 0, r.stderr[-3000:] + ign[-2000:]
    if max(trainer_done) > resume_at:
        assert f"past step {resume_at}" in ign, ign[-2000:]
    rows = [json.loads(l) for l in (rt / "tensorboard" / "actor_train-0" / "metrics.jsonl").read_text().splitlines()]
    # the resumed run's first step follows the resume point
    assert rows[-1]["step"] > resume_at and rows[len(rows) - 1]["step"] <= 3, rows
