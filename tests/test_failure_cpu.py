"""Failure detection without a GPU fault: every failure is made on the host (CPU only).

* a gloo rank that exits before a collective: the surviving rank's collective ends with an error within the
  process group's timeout instead of hanging;
* a readiness wait whose dependency died fails at once (liveness probe); one that never becomes ready times out;
* a participant whose checkpoint commit marker is missing (a shard written but never committed) moves the resume
  point back to the newest step that every participant committed;
* the engine client against a server that is down retries a bounded number of times and then raises; against a
  server that fails twice it succeeds on the third attempt; a server returning non-finite log-probs is rejected;
  an aborted generation is continued from where it stopped;
* a launcher killed with SIGKILL takes torchrun, the ignitors and the engine servers down with it.
"""

import asyncio
import json
import math
import os
import socket
import threading
import time
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer

import pytest
import torch.multiprocessing as mp


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    import datetime

    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
        x = torch.ones(4)
        dist.all_reduce(x)  # both ranks take part once
        if rank == 1:
            q.put((rank, "left"))
            q.close()
            q.join_thread()  # the message is out before the process ends
            os._exit(0)  # leaves between steps, without destroying the group
        t0 = time.monotonic()
        try:
            dist.all_reduce(x)  # the peer never arrives
            q.put((rank, "no error"))
        except Exception as e:  # noqa: BLE001 - any error is the expected outcome
            q.put((rank, f"error after {time.monotonic() - t0:.1f}s: {type(e).__name__}"))
    except Exception as e:  # noqa: BLE001
        q.put((rank, f"setup failed: {e!r}"))


def test_dead_gloo_rank_ends_the_collective_with_an_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    out = dict(q.get(timeout=120) for _ in range(2))
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert out[1] == "left", out
    assert out[0].startswith("error after"), out
    assert float(out[0].split()[2].rstrip("s:")) < 60.0, out


def test_wait_keys_fails_fast_when_the_dependency_died():
    import torch.distributed as dist

    from meshy_b200.service import bootstrap

    bootstrap.set_store(dist.HashStore())
    ctx = mp.get_context("spawn")
    child = ctx.Process(target=time.sleep, args=(0.1,))
    child.start()
    child.join()
    t0 = time.monotonic()
    with pytest.raises(RuntimeError, match="died"):
        bootstrap.wait_keys(["svc/ready"], timeout=60, interval=0.05, liveness=child.is_alive)
    assert time.monotonic() - t0 < 5
    with pytest.raises(TimeoutError):
        bootstrap.wait_keys(["svc/never"], timeout=0.3, interval=0.05)
    bootstrap.mark("svc/ready")
    bootstrap.wait_keys(["svc/ready"], timeout=1)
    bootstrap.set_store(None)


def test_resume_point_skips_an_uncommitted_shard(tmp_path):
    from meshy_b200.service.checkpoint import StateStore, resolve_resume_step

    store = StateStore(str(tmp_path))
    for step in (10, 20, 30):
        for svc in ("trainer", "rollout"):
            store.write_meta(svc, step, {"step": step})
            if not (step == 30 and svc == "rollout"):  # rollout died before committing step 30
                store.mark_complete(svc, step)
    assert store.complete_steps("rollout") == [10, 20]
    everyone = lambda step: ["trainer", "rollout"]  # noqa: E731
    assert resolve_resume_step(store, everyone) == 20
    # a participant that only joins later (cold start) does not hold the resume point back
    only_trainer_early = lambda step: ["trainer"] if step <= 10 else ["trainer", "rollout"]  # noqa: E731
    os.remove(os.path.join(store.service_dir("rollout"), "step-10.complete"))
    os.remove(os.path.join(store.service_dir("rollout"), "step-20.complete"))
    assert resolve_resume_step(store, everyone) == 0
    assert resolve_resume_step(store, only_trainer_early) == 10
    dropped = store.drop_newer_than(10)
    assert 30 in dropped.get("trainer", []) and 20 in dropped.get("trainer", [])
    assert store.complete_steps("trainer") == [10]


class _Server:
    """A /generate endpoint whose behaviour a test scripts: a list of responses consumed in order."""

    def __init__(self, script):
        self.script = list(script)
        self.calls = []
        owner = self

        class H(BaseHTTPRequestHandler):
            def do_POST(self):  # noqa: N802
                body = json.loads(self.rfile.read(int(self.headers["Content-Length"])))
                owner.calls.append(body)
                status, payload = owner.script.pop(0) if owner.script else (500, {})
                data = json.dumps(payload).encode()
                self.send_response(status)
                self.send_header("Content-Type", "application/json")
                self.send_header("Content-Length", str(len(data)))
                self.end_headers()
                self.wfile.write(data)

            def log_message(self, *a):
                pass

        self.httpd = ThreadingHTTPServer(("127.0.0.1", 0), H)
        self.url = f"http://127.0.0.1:{self.httpd.server_address[1]}"
        threading.Thread(target=self.httpd.serve_forever, daemon=True).start()

    def close(self):
        self.httpd.shutdown()
        self.httpd.server_close()


def _ok(ids, lps, reason):
    return 200, {"output_ids": ids, "meta_info": {"output_token_logprobs": [[x, 0] for x in lps],
                                                  "finish_reason": {"type": reason}, "weight_version": 3}}


def _run(coro):
    return asyncio.run(coro)


def test_engine_client_bounded_retries_and_continuation():
    pytest.importorskip("aiohttp")
    from meshy_b200.engine.rollout_client import EngineClient

    async def gen(client, prompt, params):
        try:
            return await client.generate(prompt, params)
        finally:
            if client._session is not None:
                await client._session.close()

    # nothing listening: three attempts, then the last transport error
    dead = f"http://127.0.0.1:{_port()}"
    c = EngineClient(dead, attempts=3, backoff=0.01)
    t0 = time.monotonic()
    with pytest.raises(Exception):
        _run(gen(c, [1, 2], {"max_new_tokens": 4}))
    assert time.monotonic() - t0 < 30

    # two failures, then success
    s = _Server([(500, {}), (503, {}), _ok([7, 8], [-0.5, -1.0], "length")])
    try:
        g = _run(gen(EngineClient(s.url, attempts=5, backoff=0.01), [1, 2], {"max_new_tokens": 2}))
        assert g.output_ids == [7, 8] and g.finish_reason == "length" and len(s.calls) == 3
    finally:
        s.close()

    # an aborted generation continues from the tokens it already has, with the remaining budget
    s = _Server([_ok([5], [-0.1], "abort"), _ok([6, 9], [-0.2, -0.3], "length")])
    try:
        g = _run(gen(EngineClient(s.url, attempts=2, backoff=0.01), [1, 2], {"max_new_tokens": 3}))
        assert g.output_ids == [5, 6, 9] and g.continuations == 1
        assert s.calls[1]["input_ids"] == [1, 2, 5] and s.calls[1]["sampling_params"]["max_new_tokens"] == 2
    finally:
        s.close()

    # non-finite log-probs are rejected, not passed to the trainer
    s = _Server([_ok([5], [math.nan], "stop")])
    try:
        with pytest.raises(ValueError, match="non-finite"):
            _run(gen(EngineClient(s.url, attempts=1, backoff=0.01), [1], {"max_new_tokens": 1}))
    finally:
        s.close()


@pytest.mark.timeout(240)
def test_killed_launcher_takes_its_run_down(tmp_path):
    """SIGKILL of the launcher (no chance to forward a signal) still ends torchrun, the ignitors and the
    engine servers they started: each child dies with its parent."""
    import signal
    import subprocess
    import sys

    psutil = pytest.importorskip("psutil")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, XRL_DEVICE="cpu", XRL_SMOKE_STEPS="50", PYTHONPATH=root,
               XRL_PORT_OFFSET=str(100 + (_port() % 400) * 10))
    p = subprocess.Popen([sys.executable, "-m", "meshy_b200.launch", "--recipe", "recipe.justrl_smoke",
                          "--runtime-dir", str(tmp_path / "rt"), "--master-port", str(_port())], cwd=root, env=env,
                         stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
    kids = []
    deadline = time.monotonic() + 120
    while time.monotonic() < deadline:  # until the engine servers are up (launcher > torchrun > ignitor > server)
        try:
            kids = psutil.Process(p.pid).children(recursive=True)
        except psutil.NoSuchProcess:
            break
        if sum("rollout.server" in " ".join(k.cmdline()) for k in kids if k.is_running()) >= 2:
            break
        time.sleep(1)
    assert len(kids) >= 4, [" ".join(k.cmdline()) for k in kids]
    p.send_signal(signal.SIGKILL)
    p.wait()
    gone, alive = psutil.wait_procs(kids, timeout=60)
    try:
        assert not alive, [" ".join(k.cmdline()) for k in alive]
    finally:
        for k in alive:
            k.kill()
