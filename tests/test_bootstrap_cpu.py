"""Readiness markers through the bootstrap store (CPU): round trip and a timeout that names the missing service,
markers namespaced per run directory, and a marker published by a child process -- which shares only the
inherited store address, no filesystem path -- observed by the parent."""

import multiprocessing as mp

import pytest


def _child_marks(root):
    from meshy_b200.service.runtime import RuntimeDir

    RuntimeDir(root).mark_ready("inference-0")


def test_markers(tmp_path):
    import torch.distributed as dist

    from meshy_b200.service import bootstrap
    from meshy_b200.service.runtime import RuntimeDir

    bootstrap.set_store(dist.HashStore())
    try:
        rt = RuntimeDir(str(tmp_path / "run_a"))
        assert not rt.is_ready("inference-0")
        rt.mark_ready("inference-0")
        assert rt.is_ready("inference-0")
        rt.wait_ready(["inference-0"], timeout=5)
        with pytest.raises(TimeoutError, match="training-0"):
            rt.wait_ready(["inference-0", "training-0"], timeout=0.5, interval=0.1)
        assert not RuntimeDir(str(tmp_path / "run_b")).is_ready("inference-0")  # another run, another namespace
    finally:
        bootstrap.set_store(None)


def test_marker_crosses_process_boundary(tmp_path, monkeypatch):
    from meshy_b200.service import bootstrap
    from meshy_b200.service.runtime import RuntimeDir

    for k in (bootstrap.ADDR_ENV, bootstrap.PORT_ENV):  # the store's address is restored after the test
        monkeypatch.delenv(k, raising=False)
    bootstrap.host_store("127.0.0.1", 0, timeout=60)
    try:
        root = str(tmp_path / "run")
        p = mp.get_context("spawn").Process(target=_child_marks, args=(root,))
        p.start()
        RuntimeDir(root).wait_ready(["inference-0"], timeout=120, interval=0.1, liveness=lambda: True)
        p.join(timeout=60)
        assert p.exitcode == 0
    finally:
        bootstrap.set_store(None)
