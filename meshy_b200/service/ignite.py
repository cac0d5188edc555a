"""Card-level SPMD ignitor: one process per GPU card under a single ``torchrun``.

Behaviour of the reference's ignitor (``meshy/service/ignite.py:66-310``):

1. join a gloo group over all cards (no CUDA context in the ignitor: the card
   is handed back and forth between colocated engines);
2. agree on the runtime directory (rank 0 picks, everybody receives it);
3. make sure the bootstrap store and the column store (data plane) exist:
   the launcher normally hosts both and exports their addresses; under a bare
   ``torchrun -m recipe.x`` rank 0 hosts them itself;
4. all-gather the card list and derive the topology (a pure function, so
   every rank computes the same one);
5. decide fresh-vs-resume once: reusing a runtime dir that holds checkpoints
   without ``--resume`` is an error; with ``--resume`` the resume step is the
   newest step every participant completed, shards above it are dropped and
   ``XRL_RESUME_STEP`` is published for the services;
6. for every GPU service on this card, in dependency order: wait for its
   ``wait_until`` groups' readiness markers, ignite, wait until ready (which
   publishes its own marker);
7. barrier, then rank 0 issues each colocation ring's genesis grant;
8. rank 0 starts the CPU services (rollout) the same gated way;
9. join the children (ranks without a local process idle so the torchrun
   group stays uniform).
"""

from __future__ import annotations

import logging
import os
import socket
import time

from . import bootstrap
from .base import GPU, ServiceGroup, redirect_output
from .registry import resolve_service
from .runtime import RuntimeDir
from .topology import ServiceInfo, Topology, build_topology

log = logging.getLogger(__name__)
TQ_KEY = "xrl/tq_endpoint"
SHUTDOWN_KEY = "xrl/shutdown"


def _exitcode(svc) -> int:
    p = getattr(svc, "proc", None)
    if p is None:
        return 0
    code = p.exitcode if hasattr(p, "exitcode") else p.returncode
    return 0 if code is None else abs(int(code))


def _world() -> tuple[int, int]:
    return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))


def _discover_host() -> str:
    rank, world = _world()
    if world == 1:
        return "127.0.0.1"
    master = os.environ.get("MASTER_ADDR", "127.0.0.1")
    if master in ("127.0.0.1", "localhost"):
        return "127.0.0.1"
    try:
        with socket.socket(socket.AF_INET, socket.SOCK_DGRAM) as s:
            s.connect((master, int(os.environ.get("MASTER_PORT", "29500"))))
            return s.getsockname()[0]
    except OSError:
        return "127.0.0.1"


def discover_gpus() -> list[GPU]:
    rank, world = _world()
    me = GPU(global_rank=rank, host=_discover_host(), local_rank=int(os.environ.get("LOCAL_RANK", "0")),
             node_rank=int(os.environ.get("GROUP_RANK", "0")))
    if world == 1:
        return [me]
    import torch.distributed as dist

    out: list = [None] * world
    dist.all_gather_object(out, me)
    return sorted(out, key=lambda g: g.global_rank)


class Ignitor:
    def __init__(self, service_groups: list[ServiceGroup], colocations: list | None = None):
        self.service_groups = list(service_groups)
        self.colocations = list(colocations or [])
        self.services: list = []
        self.runtime: RuntimeDir | None = None
        self.topology: Topology | None = None
        self._tq_server = None

    # ------------------------------------------------------------------ setup
    def _init_group(self) -> None:
        rank, world = _world()
        if world > 1:
            import torch.distributed as dist

            if not dist.is_initialized():
                dist.init_process_group("gloo")

    def _broadcast(self, obj):
        rank, world = _world()
        if world == 1:
            return obj
        import torch.distributed as dist

        box = [obj]
        dist.broadcast_object_list(box, src=0)
        return box[0]

    def _resolve_runtime(self) -> RuntimeDir:
        rank, _ = _world()
        root = os.environ.get("XRL_RUNTIME_DIR")
        if not root:
            root = os.path.abspath(os.path.join(".xrl_runtime", time.strftime("%Y%m%d-%H%M%S"))) if rank == 0 else None
            root = self._broadcast(root)
        os.environ["XRL_RUNTIME_DIR"] = root
        return RuntimeDir(root)

    def _ensure_bootstrap(self) -> None:
        rank, world = _world()
        if os.environ.get(bootstrap.ADDR_ENV) and os.environ.get(bootstrap.PORT_ENV):
            bootstrap.get_store()
            return
        # bare torchrun: rank 0 hosts next to the rendezvous port
        host = os.environ.get("MASTER_ADDR", "127.0.0.1")
        port = int(os.environ.get("MASTER_PORT", "29500")) + 1
        if rank == 0:
            bootstrap.host_store(host if world > 1 else "127.0.0.1", port)
        self._broadcast(None)  # rank 0's store is listening before anyone connects
        if rank != 0:
            os.environ[bootstrap.ADDR_ENV] = host
            os.environ[bootstrap.PORT_ENV] = str(port)
            bootstrap.get_store()

    def _ensure_data_plane(self) -> None:
        rank, _ = _world()
        if os.environ.get("XRL_TQ_ENDPOINTS"):
            return
        store = bootstrap.get_store()
        if rank == 0:
            from ..tq.server import ColumnStoreServer

            host = "0.0.0.0" if _world()[1] > 1 else "127.0.0.1"
            self._tq_server = ColumnStoreServer(host, 0)
            self._tq_server.start_background()
            ep = self._tq_server.endpoint
            if host == "0.0.0.0":
                ep = ep.replace("0.0.0.0", _discover_host())
            store.set(TQ_KEY, ep)
        store.wait([TQ_KEY])
        os.environ["XRL_TQ_ENDPOINTS"] = store.get(TQ_KEY).decode()

    # ------------------------------------------------------------------ run
    def run(self) -> None:
        self._init_group()
        rank, world = _world()
        self.runtime = self._resolve_runtime()
        redirect_output(self.runtime.process_log_path("ignitor", rank))
        logging.basicConfig(level=logging.INFO, format="%(asctime)s ignitor %(levelname)s %(message)s")
        self._ensure_bootstrap()
        self._ensure_data_plane()
        gpus = discover_gpus()
        self.topology = build_topology(self.service_groups, gpus, self.colocations)
        self.check_resume(self.topology)
        my_gpu = next(g for g in gpus if g.global_rank == rank)
        for info in self.topology.local_services(rank):
            svc = self._build(info, my_gpu)
            self._gate_and_start(svc, info)
            self.services.append(svc)
        if self.colocations:
            if world > 1:
                import torch.distributed as dist

                dist.barrier()
            if rank == 0:
                self.issue_genesis()
        if rank == 0:
            for info in self.topology.cpu_services():
                svc = self._build(info, None)
                self._gate_and_start(svc, info)
                self.services.append(svc)
        log.info("rank %d ready: %s", rank, [s.name for s in self.services])
        rc = self.join()
        if rc:
            raise SystemExit(rc)

    def check_resume(self, topology: Topology) -> int:
        from .checkpoint import RESUME_STEP_ENV, resolve_resume_step, resume_requested

        store = self.runtime.state_store()
        os.environ[RESUME_STEP_ENV] = "0"
        policy = topology.checkpoint_config()
        if policy is None:
            if store.has_any_shard() and resume_requested():
                raise ValueError(f"--resume was passed but no service enables checkpointing, so {store.root} "
                                 "cannot be adopted; set GlobalCheckpointConfig(enabled=True)")
            return 0
        if not store.has_any_shard():
            return 0
        if not resume_requested():
            raise ValueError(f"runtime directory {self.runtime.root} already holds global checkpoints but --resume "
                             "was not passed: pass --resume to continue that run, or use a fresh --runtime-dir")
        step = resolve_resume_step(store, topology.checkpoint_participants)
        if step <= 0:
            raise ValueError(f"--resume was passed but no step of {store.root} is complete across every "
                             "participant; start fresh with a new --runtime-dir")
        os.environ[RESUME_STEP_ENV] = str(step)
        if _world()[0] == 0:
            for svc, stale in store.drop_newer_than(step).items():
                log.info("resume: dropped %s shard(s) %s past step %d", svc, stale, step)
        return step

    def _build(self, info: ServiceInfo, my_gpu: GPU | None):
        if info.config is None:
            raise ValueError(f"service {info.name!r} has no ServiceConfig")
        svc = resolve_service(info.config).from_info(info, self.topology, self.runtime, my_gpu)
        svc.configure_colocation()
        return svc

    def _gate_and_start(self, svc, info: ServiceInfo) -> None:
        deps = self.topology.dependency_names(info)
        if deps:
            log.info("%s waits for %s", info.name, deps)
            self.runtime.wait_ready(deps)
        log.info("igniting %s (%s)", info.name, info.role)
        svc.ignite()
        svc.wait_for_ready()

    def issue_genesis(self) -> None:
        from ..tq.client import connect
        from .colocation import StoreLedger, issue_genesis

        for ring in self.colocations:
            client = connect(os.environ.get("XRL_TQ_ENDPOINTS"))
            try:
                issue_genesis(ring, StoreLedger(client, ring.group_id))
            finally:
                client.close()

    def join(self, poll: float = 1.0) -> int:
        """Wait for the run to end.

        The run ends when rank 0's CPU services (the rollout driver) have all
        exited: rank 0 then publishes ``SHUTDOWN_KEY`` and every ignitor
        terminates its local engines.  A local engine that dies first ends the
        run the same way (its exit code is returned).
        """
        rank, _ = _world()
        store = bootstrap.get_store()
        cpu = [s for s in self.services if not s.info.uses_gpu]
        rc = 0
        try:
            while True:
                if store.check([SHUTDOWN_KEY]):
                    break
                if rank == 0 and cpu and all(not s.is_alive() for s in cpu):
                    rc = max([_exitcode(s) for s in cpu] + [0])
                    store.set(SHUTDOWN_KEY, str(rc))
                    break
                dead = [s for s in self.services if s.info.uses_gpu and getattr(s, "processes", None)
                        and not s.is_alive()]
                if dead:
                    rc = _exitcode(dead[0]) or 1
                    log.error("%s exited (code %s); shutting the run down", dead[0].name, rc)
                    store.set(SHUTDOWN_KEY, str(rc))
                    break
                time.sleep(poll)
        except KeyboardInterrupt:
            pass
        self.shutdown()
        return rc

    def shutdown(self, timeout: float = 30.0) -> None:
        for s in self.services:
            s.terminate()
        deadline = time.monotonic() + timeout
        for s in self.services:
            for p in getattr(s, "processes", []):
                try:
                    if hasattr(p, "join"):
                        p.join(max(0.1, deadline - time.monotonic()))
                        if p.is_alive():
                            p.kill()
                    else:
                        p.wait(max(0.1, deadline - time.monotonic()))
                except Exception:
                    try:
                        p.kill()
                    except Exception:
                        pass
        if self._tq_server is not None:
            self._tq_server.shutdown()


__all__ = ["Ignitor", "discover_gpus"]
