"""Two ON_DEMAND members contending for one card (host only).

The JustRL-II ring is inference (FALLBACK) -> critic -> trainer. During the critic's cold start only the
critic asks for the card; the trainer joins as soon as the critic starts publishing values, so from then on
two consumers can be waiting at once. Both must get the card in turn and it must come back to the fallback
owner, with every manager thread alive. A FALLBACK owner that is handing the card over must not start a
second hand-off for the same request while it waits for the next ring member (the re-entrancy that once
left every waiter blocked).
"""

import threading
import time

from meshy_b200.service.colocation import (ColocationManager, ColocationRing, GpuRequest, MemoryLedger,
                                           SchedulingMode, issue_genesis)


def _ring(next_owner_timeout=1.0):
    return ColocationRing("actor_card", (("actor_infer", SchedulingMode.FALLBACK), ("critic", SchedulingMode.ON_DEMAND),
                                         ("actor_train", SchedulingMode.ON_DEMAND)),
                          poll_interval=0.005, next_owner_timeout=next_owner_timeout)


def _until(pred, timeout=10.0):
    end = time.monotonic() + timeout
    while not pred():
        assert time.monotonic() < end, "condition not reached"
        time.sleep(0.002)


def test_two_consumers_each_get_the_card_then_it_returns():
    ring = _ring()
    ledger = MemoryLedger()
    acquired = []
    lock = threading.Lock()

    def note(who):
        def cb(grant):
            with lock:
                acquired.append((who, grant.sequence))
        return cb

    managers = {name: ColocationManager(ring, name, lambda: ledger, on_acquire=note(name))
                for name in ("actor_infer", "critic", "actor_train")}
    for m in managers.values():
        m.start()
    try:
        issue_genesis(ring, ledger)
        _until(lambda: managers["actor_infer"].owns_gpu)
        # both consumers ask before anyone moves
        want_train = managers["actor_train"].request_gpu("actor_train:step:1")
        want_critic = managers["critic"].request_gpu("critic:window:32")
        g_critic = managers["critic"].wait_for_grant(want_critic, timeout=15)
        assert g_critic.target == "critic" and g_critic.source == "actor_infer"  # ring order after the owner
        managers["critic"].release(transition="critic-window-complete", payload_ref="/w/v0")
        g_train = managers["actor_train"].wait_for_grant(want_train, timeout=15)
        assert g_train.source == "critic" and g_train.payload_ref == "/w/v0"
        managers["actor_train"].release(transition="trained", payload_ref="/w/v1")
        _until(lambda: managers["actor_infer"].owns_gpu)
        seqs = [s for _, s in acquired]
        assert seqs == sorted(seqs) and len(set(seqs)) == len(seqs)  # one grant per sequence number, in order
        assert [w for w, _ in acquired] == ["actor_infer", "critic", "actor_train", "actor_infer"]
        assert all(m.fatal_error is None for m in managers.values())
    finally:
        for m in managers.values():
            m.stop()


def test_fallback_hand_off_is_not_re_entered_while_waiting():
    """Drive the owner's reconcile step by hand: while its transfer waits for the next ring member, a second
    consumer's request appears; the one transfer completes, to the ring's next member, and nothing recurses."""
    ring = _ring(next_owner_timeout=0.5)
    ledger = MemoryLedger()
    issue_genesis(ring, ledger)
    owner = ColocationManager(ring, "actor_infer", lambda: ledger)
    owner._reconcile(ledger.scan(), ledger)
    assert owner.owns_gpu
    entered = []
    real = owner._transfer

    def counting(*a, **kw):
        entered.append(owner._transferring)
        return real(*a, **kw)

    owner._transfer = counting
    train = GpuRequest("actor_card", "actor_train", "actor_train:step:1", time.time_ns(),
                       ring_index=ring.ring_index_for("actor_train"))
    ledger.create(train)

    def critic_arrives_later():
        time.sleep(0.1)
        ledger.create(GpuRequest("actor_card", "critic", "critic:window:1", time.time_ns(),
                                 ring_index=ring.ring_index_for("critic")))

    t = threading.Thread(target=critic_arrives_later)
    t.start()
    owner._reconcile(ledger.scan(), ledger)  # sees the trainer's request: preempt
    t.join()
    assert entered == [False]  # exactly one transfer, never entered from inside another
    assert not owner.owns_gpu and owner.owner == "critic"  # the waited-for next member wins
    owner._reconcile(ledger.scan(), ledger)  # later passes do not start another hand-off
    assert entered == [False]
