"""Colocation token ring over in-memory and column-store ledgers (host only)."""

import threading
import time

import pytest

from meshy_b200.service.colocation import (ColocationManager, ColocationRing, MemoryLedger, SchedulingMode,
                                           StoreLedger, issue_genesis)


def _ring(timeout=0.2):
    return ColocationRing("card", (("infer", SchedulingMode.FALLBACK), ("train", SchedulingMode.ON_DEMAND)),
                          poll_interval=0.02, next_owner_timeout=timeout)


@pytest.mark.parametrize("kind", ["memory", "store"])
def test_fallback_preempt_and_return(kind):
    ring = _ring()
    if kind == "memory":
        ledger = MemoryLedger()
        factory = lambda: ledger  # noqa: E731
    else:
        from meshy_b200.tq import LocalClient

        client = LocalClient()
        ledger = StoreLedger(client, ring.group_id)
        factory = lambda: StoreLedger(client, ring.group_id)  # noqa: E731
    events = []
    issue_genesis(ring, ledger)
    inf = ColocationManager(ring, "infer", factory, on_acquire=lambda g: events.append(("infer+", g.sequence)),
                            on_release=lambda t: events.append(("infer-", t)))
    tr = ColocationManager(ring, "train", factory, on_acquire=lambda g: events.append(("train+", g.sequence)),
                           on_release=lambda t: events.append(("train-", t)))
    inf.start()
    tr.start()
    try:
        deadline = time.time() + 5
        while not inf.owns_gpu and time.time() < deadline:
            time.sleep(0.01)
        assert inf.owns_gpu
        req = tr.request_gpu(payload_ref=None)
        g = tr.wait_for_grant(req, timeout=5)
        assert g.target == "train" and g.source == "infer" and g.sequence == 1 and g.transition == "preempt"
        assert ("infer-", "train") in events
        tr.release(transition="done", payload_ref="/weights/v1")
        deadline = time.time() + 5
        while not inf.owns_gpu and time.time() < deadline:
            time.sleep(0.01)
        assert inf.owns_gpu and not tr.owns_gpu
        assert [e for e in events if e[0] == "infer+"][-1][1] == 2
    finally:
        inf.stop()
        tr.stop()


def test_non_contiguous_grant_is_fatal():
    ring = _ring()
    ledger = MemoryLedger()
    issue_genesis(ring, ledger)
    from meshy_b200.service.colocation import GpuGrant, GpuRequest

    bad = GpuRequest("card", "train", "x", 1, kind=SchedulingMode.ON_DEMAND)
    ledger.create(bad)
    ledger.grant("x", GpuGrant("card", 5, "infer", "train", "x"))
    m = ColocationManager(ring, "train", lambda: ledger)
    m.start()
    deadline = time.time() + 3
    while m.fatal_error is None and time.time() < deadline:
        time.sleep(0.01)
    assert isinstance(m.fatal_error, RuntimeError)
    with pytest.raises(RuntimeError):
        m.request_gpu()


def test_ring_validation():
    with pytest.raises(ValueError):
        ColocationRing("g", (("a", "fallback"),))
    with pytest.raises(ValueError):
        ColocationRing("g", (("a", "fallback"), ("a", "on_demand")))
