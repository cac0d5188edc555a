"""Global checkpoint policy and state store (CPU): when a checkpoint is due, retention limits, the commit marker
as the only proof of a shard, payload sidecars, the resume point as the newest step every participant committed,
pruning, and clearing the tail newer than the resume point after a crash."""

import os

import pytest

from meshy_b200.config import GlobalCheckpointConfig
from meshy_b200.service.checkpoint import StateStore, resolve_resume_step


def _shard(store, svc, step, payload=None, commit=True):
    os.makedirs(store.shard_dir(svc, step), exist_ok=True)
    store.write_meta(svc, step, payload or {})
    if commit:
        store.mark_complete(svc, step)


def test_policy():
    p = GlobalCheckpointConfig(enabled=True, interval=10, keep_latest_k=2)
    assert not p.due(0) and not p.due(9) and p.due(10) and p.due(20)
    assert not GlobalCheckpointConfig(enabled=False, interval=1).due(7)
    with pytest.raises(ValueError):
        GlobalCheckpointConfig(enabled=True, keep_latest_k=1)
    with pytest.raises(ValueError):
        GlobalCheckpointConfig(enabled=True, interval=0)
    assert GlobalCheckpointConfig.coerce({"enabled": True, "interval": 4, "keep_latest_k": 2}) == \
        GlobalCheckpointConfig(enabled=True, interval=4, keep_latest_k=2)
    assert GlobalCheckpointConfig.coerce(p) is p
    assert GlobalCheckpointConfig.coerce(None) == GlobalCheckpointConfig()


def test_marker_payload_and_empty_dir(tmp_path):
    store = StateStore(str(tmp_path / "state"))
    assert store.known_services() == [] and not store.has_any_shard()
    _shard(store, "critic-0", 10, commit=False)
    assert store.complete_steps("critic-0") == [] and not store.is_complete("critic-0", 10)
    store.mark_complete("critic-0", 10)
    assert store.complete_steps("critic-0") == [10]
    _shard(store, "rollout-0", 20, {"epoch": 0, "dataset_index": 960})
    assert store.payload("rollout-0", 20) == {"epoch": 0, "dataset_index": 960}
    assert store.payload("rollout-0", 30) == {}


def test_resume_point(tmp_path):
    store = StateStore(str(tmp_path))
    for step in (10, 20, 30):
        _shard(store, "actor_train-0", step)
    for step in (10, 20):
        _shard(store, "rollout-0", step)
    _shard(store, "rollout-0", 30, commit=False)  # crashed while writing step 30
    both = lambda step: ("actor_train-0", "rollout-0")  # noqa: E731
    assert resolve_resume_step(store, both) == 20
    store2 = StateStore(str(tmp_path / "other"))
    _shard(store2, "actor_train-0", 10)
    _shard(store2, "rollout-0", 20)
    assert resolve_resume_step(store2, both) == 0  # no common step: fresh start


def test_prune_and_drop_tail(tmp_path):
    store = StateStore(str(tmp_path))
    for step in (10, 20, 30, 40):
        _shard(store, "critic-0", step)
    assert store.prune("critic-0", 2) == [10, 20]
    assert store.complete_steps("critic-0") == [30, 40]
    assert not os.path.exists(store.shard_dir("critic-0", 10)) and not os.path.exists(store.meta_path("critic-0", 10))
    assert os.path.isdir(store.shard_dir("critic-0", 40))
    for svc in ("a-0", "b-0"):
        for step in (10, 20, 30):
            _shard(store, svc, step)
    assert store.drop_newer_than(20) == {"a-0": [30], "b-0": [30], "critic-0": [30, 40]}
    assert store.complete_steps("a-0") == [10, 20] and store.complete_steps("critic-0") == []
