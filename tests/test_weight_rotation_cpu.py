"""Rotation of exported weight versions (``weights/{service}/v{N}``) and runtime directory overrides (CPU).

Old versions are pruned to the newest k, except any version a retained global checkpoint names (a resumed
inference server boots from that path); the version just written always survives; k = 0 turns rotation off.
Artifact directories follow the ``XRL_*`` environment overrides and default under the run root."""

import os

from meshy_b200.engine.trainer import TrainerEngine
from meshy_b200.service.runtime import RuntimeDir


def _pruner(runtime, keep, name="actor_train-0"):
    eng = object.__new__(TrainerEngine)  # the pruning surface only: no process group, no model
    eng.runtime, eng.weights_keep_latest_k, eng.service_name = runtime, keep, name
    return eng


def _export(runtime, name, v):
    path = runtime.checkpoint_path(name, v)
    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "model.safetensors"), "w") as f:
        f.write("x")


def _versions(runtime, name="actor_train-0"):
    return sorted(int(d[1:]) for d in os.listdir(runtime.weights_dir(name)) if d.startswith("v"))


def _runtime(tmp_path):
    return RuntimeDir(str(tmp_path / "run"), checkpoint_dir=str(tmp_path / "weights"), state_dir=str(tmp_path / "state"))


def test_keeps_newest_k_and_protected_versions(tmp_path):
    rt = _runtime(tmp_path)
    for v in range(1, 9):
        _export(rt, "actor_train-0", v)
    assert TrainerEngine.prune_weights(_pruner(rt, 3)) == [1, 2, 3, 4, 5]
    assert _versions(rt) == [6, 7, 8]
    rt2 = _runtime(tmp_path / "b")
    store = rt2.state_store()
    for v in range(1, 9):
        _export(rt2, "actor_train-0", v)
    for step, v in ((12, 2), (15, 5)):
        store.write_meta("actor_train-0", step, {"weight_version": v})
        store.mark_complete("actor_train-0", step)
    TrainerEngine.prune_weights(_pruner(rt2, 2))
    assert _versions(rt2) == [2, 5, 7, 8]


def test_tiny_keep_and_rotation_off(tmp_path):
    rt = _runtime(tmp_path)
    for v in (1, 2, 3):
        _export(rt, "actor_train-0", v)
    TrainerEngine.prune_weights(_pruner(rt, 1))
    assert _versions(rt) == [3]
    for v in (4, 5):
        _export(rt, "actor_train-0", v)
    assert TrainerEngine.prune_weights(_pruner(rt, 0)) == []
    assert _versions(rt) == [3, 4, 5]
    assert TrainerEngine.prune_weights(_pruner(_runtime(tmp_path / "empty"), 2)) == []  # nothing exported yet


def test_runtime_dirs_follow_overrides(tmp_path, monkeypatch):
    for k in ("XRL_CHECKPOINT_DIR", "XRL_STATE_DIR", "XRL_LOG_DIR", "XRL_TENSORBOARD_DIR", "XRL_TRAJECTORY_DIR"):
        monkeypatch.delenv(k, raising=False)
    rt = RuntimeDir(str(tmp_path / "root"))
    assert rt.checkpoint_dir == str(tmp_path / "root" / "weights") and rt.state_dir == str(tmp_path / "root" / "state")
    assert rt.log_dir == str(tmp_path / "root" / "logs") and rt.trajectory_dir == str(tmp_path / "root")
    monkeypatch.setenv("XRL_CHECKPOINT_DIR", str(tmp_path / "w"))
    monkeypatch.setenv("XRL_STATE_DIR", str(tmp_path / "s"))
    monkeypatch.setenv("XRL_TENSORBOARD_DIR", str(tmp_path / "tb"))
    rt = RuntimeDir(str(tmp_path / "root"))
    assert rt.checkpoint_dir == str(tmp_path / "w") and rt.state_dir == str(tmp_path / "s")
    assert rt.tensorboard_dir == str(tmp_path / "tb")
    assert rt.checkpoint_path("svc", 3) == str(tmp_path / "w" / "svc" / "v3")
