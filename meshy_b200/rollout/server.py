"""HTTP front end of the rollout engine (SGLang-compatible management API).

Routes (the subset of SGLang's API the reference drives, ``meshy/engine/sglang.py``):

* ``POST /generate`` ``{input_ids, sampling_params, return_logprob}`` →
  ``{output_ids, meta_info: {finish_reason: {type}, output_token_logprobs:
  [[lp, id, null], ...], weight_version}}``
* ``GET /health``, ``GET /health_generate``, ``GET /v1/loads``,
  ``GET /get_model_info``
* ``POST /pause_generation {mode: "abort"|"wait"}``, ``POST /continue_generation``
* ``POST /release_memory_occupation {tags}``, ``POST /resume_memory_occupation {tags}``
* ``POST /update_weights_from_disk {model_path, weight_version?}``
* ``POST /update_weights_from_ipc {handle, numel, weight_version}`` — device
  path: the trainer exports its flat bf16/fp32 buffer as a CUDA IPC handle and
  the engine copies it with one device-to-device cast (same node).

:class:`EngineRunner` owns the engine's scheduling thread; HTTP handlers and
:class:`~meshy_b200.engine.rollout_client.LocalEngineClient` both submit to it.

    python -m meshy_b200.rollout.server --model qwen2_5_math:R1-Distill-1.5B --port 30000
"""

from __future__ import annotations

import argparse
import asyncio
import logging
import threading
import time
from typing import Any

log = logging.getLogger(__name__)


class EngineRunner:
    def __init__(self, engine):
        self.engine = engine
        self._futs: dict[Any, tuple[asyncio.AbstractEventLoop, asyncio.Future]] = {}
        self._sync: dict[Any, threading.Event] = {}
        self._wake = threading.Event()
        self._stop = threading.Event()
        self._lock = threading.Lock()
        self.thread = threading.Thread(target=self._loop, name="engine-runner", daemon=True)
        self.thread.start()

    def _loop(self):
        eng = self.engine
        while not self._stop.is_set():
            if eng.paused or not eng.has_work() or eng.kv is None:
                self._wake.wait(0.05)
                self._wake.clear()
                self._deliver()
                continue
            try:
                eng.step()
            except Exception:  # keep serving; fail the requests in flight
                log.exception("engine step failed")
                for g in eng.abort_all():
                    g.finish_reason = "abort"
            self._deliver()

    def _deliver(self):
        eng = self.engine
        with self._lock:
            done = [rid for rid in list(self._futs) + list(self._sync) if rid in eng.finished]
            for rid in done:
                gen = eng.finished.pop(rid)
                if rid in self._futs:
                    loop, fut = self._futs.pop(rid)
                    loop.call_soon_threadsafe(lambda f=fut, g=gen: f.done() or f.set_result(g))
                else:
                    ev = self._sync.pop(rid)
                    ev.gen = gen
                    ev.set()

    async def generate(self, prompt, params: dict):
        loop = asyncio.get_running_loop()
        fut = loop.create_future()
        rid = self._submit(prompt, params)
        with self._lock:
            self._futs[rid] = (loop, fut)
        self._wake.set()
        return await fut

    def generate_sync(self, prompt, params: dict, timeout: float | None = None):
        ev = threading.Event()
        rid = self._submit(prompt, params)
        with self._lock:
            self._sync[rid] = ev
        self._wake.set()
        if not ev.wait(timeout):
            raise TimeoutError("generation timed out")
        return ev.gen

    def _submit(self, prompt, params: dict):
        return self.engine.submit(prompt, int(params.get("max_new_tokens", 16384)),
                                  temperature=float(params.get("temperature", 1.0)),
                                  top_k=int(params.get("top_k", -1)), top_p=float(params.get("top_p", 1.0)),
                                  ignore_eos=bool(params.get("ignore_eos", False)))

    def pause(self, mode: str = "abort") -> None:
        self.engine.pause()
        if mode == "abort":
            with self.engine.lock:
                self.engine.abort_all()
        self._deliver()

    def resume(self) -> None:
        self.engine.resume()
        self._wake.set()

    def shutdown(self) -> None:
        self._stop.set()
        self._wake.set()
        self.thread.join(timeout=5)


def build_app(runner: EngineRunner, model_name: str = ""):
    from aiohttp import web

    eng = runner.engine

    async def generate(req):
        body = await req.json()
        params = dict(body.get("sampling_params") or {})
        gen = await runner.generate(list(body["input_ids"]), params)
        out = {"output_ids": gen.output_ids,
               "meta_info": {"finish_reason": {"type": gen.finish_reason},
                             "completion_tokens": len(gen.output_ids), "weight_version": gen.weight_version}}
        if body.get("return_logprob", False):
            out["meta_info"]["output_token_logprobs"] = [[lp, t, None] for lp, t in
                                                        zip(gen.output_logprobs, gen.output_ids)]
        return web.json_response(out)

    async def health(req):
        return web.Response(text="ok")

    async def loads(req):
        return web.json_response({"loads": [eng.loads()]})

    async def info(req):
        out = {"model_path": model_name, "weight_version": eng.weight_version, "max_running": eng.max_running}
        if eng.cuda:
            from .weight_sync import device_uuid

            out["gpu_uuid"] = device_uuid(eng.device)
        return web.json_response(out)

    async def pause(req):
        body = await req.json() if req.can_read_body else {}
        await asyncio.to_thread(runner.pause, body.get("mode", "abort"))
        return web.json_response({"ok": True})

    async def cont(req):
        runner.resume()
        return web.json_response({"ok": True})

    async def release(req):
        body = await req.json() if req.can_read_body else {}
        await asyncio.to_thread(eng.release_memory, tuple(body.get("tags") or ("kv_cache", "weights")))
        return web.json_response({"ok": True})

    async def resume_mem(req):
        body = await req.json() if req.can_read_body else {}
        await asyncio.to_thread(eng.resume_memory, tuple(body.get("tags") or ("kv_cache", "weights")))
        runner._wake.set()
        return web.json_response({"ok": True})

    async def load_disk(req):
        body = await req.json()
        t0 = time.perf_counter()
        await asyncio.to_thread(eng.update_weights_from_disk, body["model_path"], body.get("weight_version"))
        return web.json_response({"ok": True, "seconds": time.perf_counter() - t0})

    async def load_ipc(req):
        """``{handle}``: one exported buffer; ``{handles: {gpu_uuid: handle}}``: one per trainer rank, of
        which this server maps the one exported on its own GPU (see ``weight_sync.pick_handle``)."""
        body = await req.json()
        from .weight_sync import open_ipc_flat

        t0 = time.perf_counter()
        local = True

        def do():
            nonlocal local
            if body.get("handle") is None:  # one handle per trainer rank: every engine rank maps its own GPU's
                local = eng.update_weights_from_ipc(body["handles"], body.get("weight_version"))
                return
            if getattr(eng, "tp", 1) > 1:
                raise ValueError("a tensor-parallel replica needs the per-GPU handle set ('handles')")
            src = open_ipc_flat(body["handle"], body.get("gpu_uuid"))
            eng.update_weights_from_flat(src, body.get("weight_version"))
            if eng.cuda:
                import torch

                torch.cuda.synchronize(eng.device)
            del src

        await asyncio.to_thread(do)
        dt = time.perf_counter() - t0
        print(f"[weight-sync] ipc version {body.get('weight_version')} local={local} {dt * 1e3:.2f} ms", flush=True)
        return web.json_response({"ok": True, "seconds": dt, "local": local})

    app = web.Application(client_max_size=1 << 30)
    app.add_routes([
        web.post("/generate", generate), web.get("/health", health), web.get("/health_generate", health),
        web.get("/v1/loads", loads), web.get("/get_model_info", info), web.post("/pause_generation", pause),
        web.post("/continue_generation", cont), web.post("/release_memory_occupation", release),
        web.post("/resume_memory_occupation", resume_mem), web.post("/update_weights_from_disk", load_disk),
        web.post("/update_weights_from_ipc", load_ipc),
    ])
    return app


def serve(engine, host: str, port: int, model_name: str = "") -> None:
    from aiohttp import web

    runner = EngineRunner(engine)
    web.run_app(build_app(runner, model_name), host=host, port=port, print=None, access_log=None)


def main(argv=None):
    p = argparse.ArgumentParser(description="meshy_b200 rollout engine server")
    p.add_argument("--model", required=True, help="model_name:flavor of the registry")
    p.add_argument("--model-path", default=None, help="HF checkpoint dir to load (random init when absent)")
    p.add_argument("--host", default="127.0.0.1")
    p.add_argument("--port", type=int, default=30000)
    p.add_argument("--device", default="cuda")
    p.add_argument("--max-running", type=int, default=256)
    p.add_argument("--max-total-tokens", type=int, default=None)
    p.add_argument("--max-seq-len", type=int, default=None)
    p.add_argument("--mem-fraction", type=float, default=0.5)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--eos", type=int, nargs="*", default=[])
    p.add_argument("--tp-size", type=int, default=1, help="tensor-parallel degree of this replica")
    p.add_argument("--ep-size", type=int, default=1, help="expert-parallel degree of this replica")
    p.add_argument("--dist-port", type=int, default=0, help="rendezvous port of the TP ranks (0: free port)")
    p.add_argument("--nnodes", type=int, default=1, help="nodes the replica's TP ranks span")
    p.add_argument("--node-rank", type=int, default=0, help="this node's index among them (0 serves HTTP)")
    p.add_argument("--dist-init-addr", default="", help="host:port of the TP rendezvous (multi-node replicas)")
    a = p.parse_args(argv)
    if a.ep_size > 1 and a.ep_size != a.tp_size:
        raise SystemExit("--ep-size splits the MoE experts over the ranks of a tensor-parallel replica: it must "
                         "equal --tp-size (or be 1: every rank keeps every expert)")
    if a.nnodes < 1 or a.tp_size % a.nnodes or not 0 <= a.node_rank < a.nnodes:
        raise SystemExit(f"--tp-size {a.tp_size} must split evenly over --nnodes {a.nnodes}, and --node-rank "
                         f"must be below it")
    if a.nnodes > 1 and not a.dist_init_addr:
        raise SystemExit("a replica over several nodes needs --dist-init-addr host:port (node 0's address)")
    if a.tp_size > 1:
        return _serve_tp(a) if a.node_rank == 0 else _serve_tp_node(a)
    eng = _build_engine(a)
    if a.model_path:
        eng.update_weights_from_disk(a.model_path, 0)
    serve(eng, a.host, a.port, a.model_path or a.model)


def _build_engine(a, device=None, tp_group=None):
    from ..models import get_model_args
    from .engine import RolloutEngine

    name, flavor = a.model.split(":")
    return RolloutEngine(get_model_args(name, flavor), device=device or a.device, max_running=a.max_running,
                         max_total_tokens=a.max_total_tokens, max_seq_len=a.max_seq_len,
                         mem_fraction=a.mem_fraction, seed=a.seed, eos_token_ids=a.eos, tp_group=tp_group,
                         ep=a.ep_size > 1)


def _rendezvous(a) -> tuple[str, int]:
    if a.dist_init_addr:
        host, port = a.dist_init_addr.rsplit(":", 1)
        return host, int(port)
    return "127.0.0.1", a.dist_port


def _local_ranks(a) -> range:
    """Global TP ranks run on this node: ``tp_size / nnodes`` consecutive ones, node 0 first (as SGLang's
    ``--nnodes``/``--node-rank`` place them)."""
    per = a.tp_size // a.nnodes
    return range(a.node_rank * per, (a.node_rank + 1) * per)


def _tp_rank_setup(a, rank: int):
    """Process group of one TP replica (NCCL on the GPU for the partial sums, gloo for the control channel).
    ``rank`` is the global TP rank; its GPU is the node-local index among the visible devices."""
    import os
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    host, port = _rendezvous(a)
    os.environ.update(MASTER_ADDR=host, MASTER_PORT=str(port))
    os.environ.pop("TORCHELASTIC_USE_AGENT_STORE", None)  # rank 0 hosts this rendezvous itself
    cuda = a.device.startswith("cuda")
    device = torch.device("cuda", rank - _local_ranks(a).start) if cuda else torch.device("cpu")
    kw = {"device_id": device} if cuda else {}
    if cuda:
        torch.cuda.set_device(device)
    dist.init_process_group("nccl" if cuda else "gloo", rank=rank, world_size=a.tp_size,
                            timeout=timedelta(seconds=600), **kw)
    ctrl = dist.new_group(backend="gloo") if cuda else dist.group.WORLD
    return device, dist.group.WORLD, ctrl


def _tp_follower(a, rank: int) -> None:
    from .spmd import follow

    import torch.distributed as dist

    device, group, ctrl = _tp_rank_setup(a, rank)
    eng = _build_engine(a, device=str(device), tp_group=group)
    follow(eng, ctrl)
    eng._graphs.clear()  # captured graphs hold NCCL calls: release them before the process group
    dist.destroy_process_group()


def _spawn_followers(a, ranks) -> list:
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_tp_follower, args=(a, r), daemon=True) for r in ranks]
    for p_ in procs:
        p_.start()
    return procs


def _serve_tp_node(a) -> None:
    """A further node of a multi-node replica: every local rank is a follower; the process ends when node 0's
    leader stops the replica."""
    import sys

    procs = _spawn_followers(a, _local_ranks(a))
    for p_ in procs:
        p_.join()
    bad = [p_.exitcode for p_ in procs if p_.exitcode]
    if bad:
        sys.exit(f"tensor-parallel follower exited with {bad}")


def _serve_tp(a) -> None:
    """Rank 0 serves HTTP and drives the replica's other ranks: ``tp_size / nnodes - 1`` follower processes
    here (one per further visible GPU) and, for a multi-node replica, those that the other nodes' servers
    start (``_serve_tp_node``)."""
    import socket

    from .spmd import EngineLeader

    if not a.dist_port and not a.dist_init_addr:
        with socket.socket() as s_:
            s_.bind(("127.0.0.1", 0))
            a.dist_port = s_.getsockname()[1]
    procs = _spawn_followers(a, _local_ranks(a)[1:])
    device, group, ctrl = _tp_rank_setup(a, 0)
    eng = EngineLeader(_build_engine(a, device=str(device), tp_group=group), ctrl)
    if a.model_path:
        eng.update_weights_from_disk(a.model_path, 0)
    try:
        serve(eng, a.host, a.port, a.model_path or a.model)
    finally:
        try:
            eng.stop()
        except Exception:  # noqa: BLE001 - at teardown the followers got the same signal and are gone already
            pass
        for p_ in procs:
            p_.join(timeout=30)


if __name__ == "__main__":
    main()
