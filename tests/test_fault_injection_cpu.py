"""Host-side fault injection (``meshy_b200.utils.faults``) driving the failure paths, CPU only.

* plan parsing and the proxy's semantics (raise / drop / delay / pass, repeats, playback order);
* the data-plane worker retries a read that fails twice and gives up with ``TQWorkerError`` when it fails more
  often than its retry budget;
* a colocation request whose ledger write is dropped times out for its waiter (no hang) and a new request is
  granted; a ledger that starts failing kills the manager and wakes its waiter with an error;
* the ``XRL_FAULTS`` plan reaches clients made by ``tq.client.connect``;
* a rollout server killed in the middle of a generation ends the client's call with an error in bounded time;
* a gloo rank that is stopped (SIGSTOP: alive but silent) ends the other rank's collective with an error.
"""

import asyncio
import os
import signal
import socket
import subprocess
import sys
import threading
import time

import pytest
import torch.multiprocessing as mp

from meshy_b200.utils.faults import FaultyProxy, InjectedFault, inject, parse_plan

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class _Target:
    def __init__(self):
        self.calls = []
        self.value = 7

    def f(self, x):
        self.calls.append(x)
        return x * 2

    def g(self):
        return "g"


def test_plan_parsing_and_proxy():
    plan = parse_plan("tq:get_data=raise*2,pass,put=delay0.05; ledger:create=drop")
    assert plan == {"tq": {"get_data": ["raise", "raise", "pass"], "put": ["delay0.05"]},
                    "ledger": {"create": ["drop"]}}
    for bad in ("tq", "tq:f=explode", "tq:f=delayx", ":f=raise", "tq:raise"):
        with pytest.raises(ValueError):
            parse_plan(bad)
    t = _Target()
    p = inject(t, "x", {"x": {"f": ["pass", "raise", "drop", "delay0.05"]}})
    assert isinstance(p, FaultyProxy) and p.value == 7 and p.g() == "g"
    assert p.f(1) == 2
    with pytest.raises(InjectedFault):
        p.f(2)
    assert p.f(3) is None  # dropped: the target never saw it
    t0 = time.monotonic()
    assert p.f(4) == 8 and time.monotonic() - t0 >= 0.05
    assert p.f(5) == 10 and p.pending() == 0  # the plan has played out
    assert t.calls == [1, 4, 5]
    assert p.events == [("f", "raise"), ("f", "drop"), ("f", "delay0.05")]
    assert inject(t, "other", {"x": {"f": ["raise"]}}) is t
    assert inject(t, "x", "") is t


def _tq_worker(store, plan, retries=3):
    from meshy_b200.tq import LocalClient
    from meshy_b200.worker.tq import TQInput, TQOutput, TQWorker

    class Doubler(TQWorker):
        tq_max_retries = retries
        tq_retry_interval = 0.01

        def process_tq_batch(self, samples):
            from meshy_b200.tq.client import Columns

            return {"y": Columns({"y": [s["x"] * 2 for s in samples]})}

    w = Doubler()
    w.configure_tq(input=TQInput("p", ["x"], 2, "doubler", clear_after_success=False),
                   outputs={"y": TQOutput(["y"])}, client_factory=lambda: inject(LocalClient(store), "tq", plan))
    return w


def test_tq_worker_retries_injected_read_faults():
    from meshy_b200._native import ColumnStore
    from meshy_b200.tq import LocalClient
    from meshy_b200.worker.tq import TQWorkerError

    store = ColumnStore()
    src = LocalClient(store)
    src.put({"x": [1, 2, 3, 4]}, partition_id="p")
    w = _tq_worker(store, "tq:get_data=raise*2")
    client = w._connect_tq()
    assert w.run_tq_once(client)  # two failed reads, the third succeeds
    assert w._tq_stats["errors"] == 2 and client.events == [("get_data", "raise")] * 2
    meta = src.get_meta(["x", "y"], 2, "p", mode="force_fetch", task_name="check")
    got = src.get_data(meta)
    assert sorted(got["y"]) == [2, 4]
    w = _tq_worker(store, "tq:get_data=raise*4")
    with pytest.raises(TQWorkerError, match="read phase"):
        w.run_tq_once(w._connect_tq())  # 4 failures > 1 + 3 retries


def _ring():
    from meshy_b200.service.colocation import ColocationRing, SchedulingMode

    return ColocationRing("card", (("infer", SchedulingMode.FALLBACK), ("train", SchedulingMode.ON_DEMAND)),
                          poll_interval=0.02, next_owner_timeout=0.2)


def _until(cond, timeout=5.0):
    deadline = time.time() + timeout
    while not cond() and time.time() < deadline:
        time.sleep(0.01)
    return cond()


def test_dropped_ledger_write_times_out_then_a_new_request_is_granted():
    from meshy_b200.service.colocation import ColocationManager, MemoryLedger, issue_genesis

    ring = _ring()
    ledger = MemoryLedger()
    issue_genesis(ring, ledger)
    faulty = inject(ledger, "ledger", "ledger:create=drop")
    inf = ColocationManager(ring, "infer", lambda: ledger)
    tr = ColocationManager(ring, "train", lambda: faulty)
    inf.start()
    tr.start()
    try:
        assert _until(lambda: inf.owns_gpu)
        lost = tr.request_gpu()
        t0 = time.monotonic()
        with pytest.raises(TimeoutError):
            tr.wait_for_grant(lost, timeout=0.5)  # the ledger never saw it: nobody hands the card over
        assert time.monotonic() - t0 < 2 and inf.owns_gpu
        req = tr.request_gpu()
        g = tr.wait_for_grant(req, timeout=5)
        assert g.target == "train" and g.source == "infer" and faulty.events == [("create", "drop")]
        tr.release(transition="done")
        assert _until(lambda: inf.owns_gpu)
        assert inf.fatal_error is None and tr.fatal_error is None
    finally:
        inf.stop()
        tr.stop()


def test_failing_ledger_wakes_the_waiter_with_an_error():
    from meshy_b200.service.colocation import ColocationManager, MemoryLedger, issue_genesis

    ring = _ring()
    ledger = MemoryLedger()
    issue_genesis(ring, ledger)
    faulty = FaultyProxy(ledger, {"scan": ["pass"] * 20 + ["raise"]}, "ledger")
    tr = ColocationManager(ring, "train", lambda: faulty)
    tr.start()
    try:
        req = tr.request_gpu()  # "infer" never runs: the request stays open until the ledger fails
        t0 = time.monotonic()
        with pytest.raises(RuntimeError, match="colocation manager failed"):
            tr.wait_for_grant(req, timeout=10)
        assert time.monotonic() - t0 < 5 and isinstance(tr.fatal_error, InjectedFault)
        with pytest.raises(RuntimeError):
            tr.request_gpu()
    finally:
        tr.stop()


def test_env_plan_reaches_connect(monkeypatch):
    from meshy_b200.tq.client import connect

    monkeypatch.setenv("XRL_FAULTS", "tq:num_rows=raise")
    c = connect(None)
    with pytest.raises(InjectedFault):
        c.num_rows("p")
    assert c.num_rows("p") == 0
    monkeypatch.delenv("XRL_FAULTS")
    assert not isinstance(connect(None), FaultyProxy)


def _wait_health(port, proc, timeout=120):
    import requests

    end = time.time() + timeout
    while time.time() < end:
        assert proc.poll() is None, proc.stdout.read().decode()[-3000:]
        try:
            if requests.get(f"http://127.0.0.1:{port}/health", timeout=2).ok:
                return
        except Exception:
            time.sleep(0.3)
    raise AssertionError("server did not come up")


@pytest.mark.timeout(240)
def test_server_killed_mid_generation_ends_the_call_with_an_error():
    pytest.importorskip("aiohttp")
    from meshy_b200.engine.rollout_client import EngineClient

    port = _port()
    cmd = [sys.executable, "-m", "meshy_b200.rollout.server", "--model", "qwen3:debugmodel", "--device", "cpu",
           "--port", str(port), "--max-running", "4", "--max-seq-len", "4096"]
    proc = subprocess.Popen(cmd, env=dict(os.environ, PYTHONPATH=ROOT), cwd=ROOT, stdout=subprocess.PIPE,
                            stderr=subprocess.STDOUT, start_new_session=True)
    try:
        _wait_health(port, proc)
        out = {}

        async def gen():
            c = EngineClient(f"http://127.0.0.1:{port}", attempts=3, backoff=0.1)
            try:
                await c.generate([3, 14, 15], {"max_new_tokens": 4000, "temperature": 0.0, "ignore_eos": True})
                out["result"] = "finished"
            except Exception as e:  # noqa: BLE001 - the expected outcome
                out["result"] = e
            finally:
                await c.close()

        t = threading.Thread(target=lambda: asyncio.run(gen()))
        t.start()
        time.sleep(1.0)
        assert "result" not in out, "the generation ended before the server was killed"
        os.killpg(proc.pid, signal.SIGKILL)
        t0 = time.monotonic()
        t.join(timeout=60)
        assert not t.is_alive() and time.monotonic() - t0 < 60
        assert isinstance(out["result"], Exception), out["result"]
    finally:
        if proc.poll() is None:
            os.killpg(proc.pid, signal.SIGKILL)
        proc.wait(timeout=30)


def _stopped_rank(rank, port, q):
    import datetime

    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=5))
        x = torch.ones(4)
        dist.all_reduce(x)
        if rank == 1:
            q.put((rank, os.getpid()))
            q.close()
            q.join_thread()
            os.kill(os.getpid(), signal.SIGSTOP)  # alive, holding its sockets, silent
            return
        t0 = time.monotonic()
        try:
            dist.all_reduce(x)
            q.put((rank, "no error"))
        except Exception as e:  # noqa: BLE001
            q.put((rank, f"error after {time.monotonic() - t0:.1f}s: {type(e).__name__}"))
    except Exception as e:  # noqa: BLE001
        q.put((rank, f"setup failed: {e!r}"))


@pytest.mark.timeout(120)
def test_stopped_gloo_rank_ends_the_collective_with_an_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_stopped_rank, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    try:
        res = dict(q.get(timeout=90) for _ in range(2))
        assert isinstance(res[1], int)
        assert res[0].startswith("error after"), res[0]
        assert float(res[0].split()[2].rstrip("s:")) < 30
    finally:
        for p in ps:
            if p.is_alive():
                os.kill(p.pid, signal.SIGKILL)
            p.join(timeout=30)
