"""Inference service: one native rollout-engine server per replica.

Counterpart of the reference's SGLang service (``meshy/service/inference.py:
53-312``): the master card of each replica starts
``python -m meshy_b200.rollout.server`` as a subprocess in its own session
(so its CUDA context and any ``torch.distributed`` init stay out of the
ignitor), with the recipe's ``server_args`` translated to server flags
(SGLang-style keys are accepted), waits for ``/health_generate``, and then

* colocated replicas release their KV cache and weights right away so the
  trainer sharing the card can load, and the ring's leader replica builds the
  colocation manager whose callbacks drive ``/release_memory_occupation`` /
  ``/resume_memory_occupation`` + the weight reload on every replica of the
  group;
* on resume the server boots from the checkpointed weight export of the
  resume step (``_boot_model_path``).
"""

from __future__ import annotations

import logging
import os
import signal
import subprocess
import sys
import time
from typing import Any

from .base import Service, die_with_parent

log = logging.getLogger(__name__)

_TORCHRUN_VARS = frozenset({"RANK", "LOCAL_RANK", "WORLD_SIZE", "LOCAL_WORLD_SIZE", "GROUP_RANK", "GROUP_WORLD_SIZE",
                            "ROLE_RANK", "ROLE_WORLD_SIZE", "ROLE_NAME", "MASTER_ADDR", "MASTER_PORT",
                            "TORCH_NCCL_ASYNC_ERROR_HANDLING"})

# SGLang-style server_args key -> rollout.server flag
_ARG_MAP = {
    "max_running_requests": "--max-running",
    "max_total_tokens": "--max-total-tokens",
    "context_length": "--max-seq-len",
    "max_seq_len": "--max-seq-len",
    "mem_fraction_static": "--mem-fraction",
    "mem_fraction": "--mem-fraction",
    "random_seed": "--seed",
    "tp_size": "--tp-size",
    "ep_size": "--ep-size",
}
# accepted and ignored (behaviour is built in or not applicable)
_IGNORED = {"enable_memory_saver", "attention_backend", "disable_radix_cache", "skip_tokenizer_init",
            "log_level", "dtype", "trust_remote_code", "cuda_graph_max_bs", "chunked_prefill_size",
            "enable_deterministic_inference", "schedule_policy", "disable_cuda_graph", "sampling_backend"}


def server_args_to_cli(server_args: dict[str, Any]) -> list[str]:
    out: list[str] = []
    for k, v in sorted(server_args.items()):
        if k in _IGNORED or v is None or v is False:
            continue
        flag = _ARG_MAP.get(k)
        if flag is None:
            raise ValueError(f"unsupported inference server_args key {k!r}")
        out += [flag, str(v)]
    return out


class InferenceService(Service):
    def __init__(self, info, topology, runtime, my_gpu=None):
        super().__init__(info, topology, runtime)
        rank = int(os.environ.get("RANK", "0")) if my_gpu is None else my_gpu.global_rank
        ranks = [g.global_rank for g in info.replica_gpus]
        self.rank_in_replica = ranks.index(rank) if rank in ranks else 0
        self.my_gpu = info.replica_gpus[self.rank_in_replica]
        self.is_master = self.rank_in_replica == 0
        # a replica's cards by node, in node order; the lowest global rank of each node starts that node's server
        by_node: dict[int, list] = {}
        for g in info.replica_gpus:
            by_node.setdefault(g.node_rank, []).append(g)
        self.nodes = sorted(by_node)
        self.node_gpus = sorted(by_node[self.my_gpu.node_rank], key=lambda g: g.global_rank)
        self.is_node_leader = self.my_gpu.global_rank == self.node_gpus[0].global_rank
        self.processes: list = []
        self.client = None

    @classmethod
    def from_info(cls, info, topology, runtime, my_gpu=None):
        return cls(info, topology, runtime, my_gpu)

    # ------------------------------------------------------------------ launch
    def model_spec(self) -> str:
        cfg = self.info.config
        spec = cfg.server_args.get("model", None) if isinstance(cfg.server_args, dict) else None
        return spec or os.environ.get("XRL_MODEL_SPEC") or cfg.model_path

    def _boot_model_path(self) -> str | None:
        """HF weights to boot from: the trainer's export at the resume step, else the base model."""
        from .checkpoint import run_resume_step

        cfg = self.info.config
        step = run_resume_step()
        if step > 0 and self.topology is not None:
            store = self.runtime.state_store()
            for t in self.topology.training_services():
                if store.is_complete(t.name, step):
                    v = store.payload(t.name, step).get("weight_version")
                    if v is not None:
                        path = self.runtime.checkpoint_path(t.name, int(v))
                        if os.path.isdir(path):
                            return path
        return cfg.model_path if cfg.model_path and os.path.isdir(cfg.model_path) else None

    def command(self) -> list[str]:
        cfg = self.info.config
        args = dict(cfg.server_args)
        model = args.pop("model", None) or os.environ.get("XRL_MODEL_SPEC")
        if not model:
            raise ValueError(f"{self.name}: server_args['model'] must name the architecture (e.g. "
                             "'qwen2_5_math:R1-Distill-1.5B')")
        device = os.environ.get("XRL_DEVICE", "cuda")
        cmd = [sys.executable, "-m", "meshy_b200.rollout.server", "--model", model, "--host", "0.0.0.0",
               "--port", str(self.info.endpoint_port), "--device", "cuda" if device == "cuda" else device]
        boot = self._boot_model_path()
        if boot:
            cmd += ["--model-path", boot]
        # the replica's cards set its tensor-parallel degree, whatever server_args say (as the reference's
        # SGLang launch does); a replica over several nodes rendezvouses at the master card's host
        args["tp_size"] = len(self.info.replica_gpus)
        cmd += server_args_to_cli(args)
        if len(self.nodes) > 1:
            cmd += ["--nnodes", str(len(self.nodes)), "--node-rank", str(self.nodes.index(self.my_gpu.node_rank)),
                    "--dist-init-addr", f"{self.info.replica_gpus[0].host}:{self.info.dist_port}"]
        elif len(self.info.replica_gpus) > 1:
            cmd += ["--dist-port", str(self.info.dist_port)]
        return cmd

    def ignite(self) -> None:
        if not self.is_node_leader:
            return
        # none of the ignitor's torchrun variables reach the server: with TORCHELASTIC_USE_AGENT_STORE set, a
        # tensor-parallel replica's rank 0 would wait for an agent store on its rendezvous port instead of
        # hosting it
        env = {k: v for k, v in os.environ.items()
               if k not in _TORCHRUN_VARS and not k.startswith("TORCHELASTIC_")}
        if env.get("XRL_DEVICE", "cuda") == "cuda":
            env["CUDA_VISIBLE_DEVICES"] = ",".join(str(g.local_rank) for g in self.node_gpus)
        log_path = self.runtime.process_log_path(self.name, self.rank_in_replica)
        self._log = open(log_path, "ab")
        # own session (killpg on terminate) + PR_SET_PDEATHSIG so a dead ignitor takes the server with it
        self.proc = subprocess.Popen(self.command(), stdout=self._log, stderr=subprocess.STDOUT, env=env,
                                     start_new_session=True, preexec_fn=die_with_parent)
        self.processes.append(self.proc)

    def is_alive(self) -> bool:
        return self.proc is not None and self.proc.poll() is None

    def terminate(self) -> None:
        if self.proc is not None and self.proc.poll() is None:
            try:
                os.killpg(self.proc.pid, signal.SIGTERM)
            except Exception:
                pass

    def wait_for_ready(self, timeout: float = 1800.0) -> None:
        if not self.is_master:
            return
        from ..engine.rollout_client import EngineClient

        self.client = EngineClient([self.info.endpoint])
        self.client.wait_ready(liveness=self.is_alive, timeout=timeout)
        if self.info.is_colocate or self.info.colocation is not None:
            # hand the card to the ring's trainer: memory goes back before readiness is announced
            self.client.pause_generation()
            self.client.release_memory()
        if self.info.colocation is not None and self.info.is_colocation_leader:
            self._start_ring_manager()
        self.runtime.mark_ready(self.name)
        log.info("inference %s ready at %s", self.name, self.info.endpoint)

    def _start_ring_manager(self) -> None:
        """Leader replica: one manager for the whole group; callbacks fan out to every replica."""
        from ..engine.rollout_client import EngineClient
        from ..tq.client import connect
        from .colocation import ColocationManager, StoreLedger
        from ..utils.faults import inject

        ring = self.info.colocation
        group = EngineClient([s.endpoint for s in self.topology.group(self.info.group_id)])
        ref = os.environ.get("XRL_TQ_ENDPOINTS")
        self.colocation_manager = ColocationManager(
            ring, self.info.group_id, lambda: inject(StoreLedger(connect(ref), ring.group_id), "ledger"),
            on_acquire=group.on_colocate_acquire, on_release=group.on_colocate_release)
        self.colocation_manager.start()

    def health_info(self) -> dict[str, Any]:
        return {"name": self.name, "endpoint": self.info.endpoint, "alive": self.is_alive()}


__all__ = ["InferenceService", "server_args_to_cli"]
