"""Topology: a pure function of (recipe service groups, all-gathered GPU list).

Cards are assigned in declaration order; ``colocate_with=X`` reuses X's exact
card block; ports are ``<role base> + master rank``; colocation rings are
attached and validated; checkpoint policies and critic/trainer column wiring
are checked before any process starts.  Semantics follow the reference
(``meshy/service/topology.py:233-526``) because every rank must derive the
same answer from the same inputs.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

from ..config import CRITIC_OUTPUT_FIELDS_BY_MODE, ServiceConfig
from .base import GPU, ServiceGroup


@dataclass
class ServiceInfo:
    name: str
    group_id: str
    role: str
    uses_gpu: bool
    replica_idx: int
    host: str
    endpoint_port: int
    dist_port: int
    replica_gpus: list[GPU]
    is_colocate: bool
    colocate_with: str | None
    wait_until: list[str] = field(default_factory=list)
    config: ServiceConfig | None = None
    colocation: Any = None
    is_colocation_leader: bool = False

    @property
    def endpoint(self) -> str:
        return f"http://{self.host}:{self.endpoint_port}"

    @property
    def master_rank(self) -> int:
        return self.replica_gpus[0].global_rank

    def contains_rank(self, rank: int) -> bool:
        return any(g.global_rank == rank for g in self.replica_gpus)


@dataclass
class Topology:
    services: list[ServiceInfo]

    def group(self, gid: str) -> list[ServiceInfo]:
        return [s for s in self.services if s.group_id == gid]

    def by_name(self, name: str) -> ServiceInfo:
        for s in self.services:
            if s.name == name:
                return s
        raise KeyError(f"no service named {name!r}")

    def gpu_services(self):
        return [s for s in self.services if s.uses_gpu]

    def cpu_services(self):
        return [s for s in self.services if not s.uses_gpu]

    def services_by_role(self, role: str):
        return [s for s in self.services if s.role == role]

    def inference_services(self):
        return self.services_by_role("inference")

    def training_services(self):
        return self.services_by_role("training")

    def rollout_services(self):
        return self.services_by_role("rollout")

    def inference_endpoints(self) -> list[str]:
        return [s.endpoint for s in self.inference_services()]

    def inference_targets(self) -> list[dict]:
        return [{"name": s.name, "endpoint": s.endpoint} for s in self.inference_services()]

    def trainer_endpoint(self) -> str | None:
        t = self.training_services()
        return t[0].endpoint if t else None

    def checkpointing_services(self):
        return [s for s in self.services
                if getattr(getattr(s, "config", None), "checkpoint", None) is not None and s.config.checkpoint.enabled]

    def checkpoint_config(self):
        e = self.checkpointing_services()
        return e[0].config.checkpoint if e else None

    def cold_start_windows(self) -> int:
        for s in self.services_by_role("critic"):
            return int(getattr(s.config, "cold_start_windows", 0))
        return 0

    def checkpoint_participants(self, step: int) -> tuple[str, ...]:
        """Services that must hold a shard for ``step``; the trainer is exempt during the critic cold start."""
        cold = self.cold_start_windows()
        return tuple(s.name for s in self.checkpointing_services()
                     if not (s.role == "training" and (cold < 0 or int(step) <= cold)))

    def dependency_names(self, s: ServiceInfo) -> list[str]:
        return [x.name for gid in s.wait_until for x in self.group(gid)]

    def local_services(self, rank: int) -> list[ServiceInfo]:
        return [s for s in self.gpu_services() if s.contains_rank(rank)]

    def colocated_inference_for(self, trainer: ServiceInfo):
        if trainer.colocate_with is None:
            return [], {}, []
        mine = {g.global_rank for g in trainer.replica_gpus}
        names, by_rank, eps = [], {}, []
        for inf in self.group(trainer.colocate_with):
            shared = [g.global_rank for g in inf.replica_gpus if g.global_rank in mine]
            if not shared:
                continue
            for r in shared:
                by_rank[r] = inf.name
            names.append(inf.name)
            eps.append(inf.endpoint)
        return names, by_rank, eps


def build_topology(service_groups: list[ServiceGroup], gpus: list[GPU], colocations: list | None = None) -> Topology:
    gpus = sorted(gpus, key=lambda g: g.global_rank)
    targets = {sg.colocate_with for sg in service_groups if sg.colocate_with}
    blocks: dict[str, list[GPU]] = {}
    services: list[ServiceInfo] = []
    cursor = 0
    for sg in service_groups:
        ctype = type(sg.config)
        if not sg.role or sg.role == "?":
            raise ValueError(f"ServiceConfig {ctype.__name__} must declare a role")
        if not sg.uses_gpu:
            for r in range(sg.n_replicas):
                services.append(ServiceInfo(f"{sg.id}-{r}", sg.id, sg.role, False, r, "127.0.0.1", 0, 0, [], False,
                                            None, list(sg.wait_until), sg.config))
            continue
        total = sg.n_replicas * sg.n_gpus_per_replica
        if sg.colocate_with is not None:
            if sg.colocate_with not in blocks:
                raise ValueError(f"group {sg.id!r} colocate_with={sg.colocate_with!r} which is not a GPU group "
                                 "declared earlier")
            block = blocks[sg.colocate_with]
            if len(block) != total:
                raise ValueError(f"colocate group {sg.id!r} occupies {total} cards but {sg.colocate_with!r} "
                                 f"occupies {len(block)}; they must match")
        else:
            block = gpus[cursor:cursor + total]
            if len(block) != total:
                raise ValueError(f"group {sg.id!r} needs {total} cards but only {len(block)} remain")
            cursor += total
            blocks[sg.id] = block
        colo = sg.colocate_with is not None or sg.id in targets
        if ctype.endpoint_port_base is None or ctype.dist_port_base is None:
            raise ValueError(f"GPU ServiceConfig {ctype.__name__} must declare endpoint_port_base and dist_port_base")
        for r in range(sg.n_replicas):
            rg = block[r * sg.n_gpus_per_replica:(r + 1) * sg.n_gpus_per_replica]
            m = rg[0].global_rank
            services.append(ServiceInfo(f"{sg.id}-{r}", sg.id, sg.role, True, r, rg[0].host,
                                        ctype.endpoint_port_base + m, ctype.dist_port_base + m, list(rg), colo,
                                        sg.colocate_with, list(sg.wait_until), sg.config))
    _attach_colocations(services, colocations or [])
    _validate_ports(services)
    _validate_critic_columns(services)
    _validate_checkpoint(services)
    return Topology(services)


def _validate_checkpoint(services: list[ServiceInfo]) -> None:
    enabled = [s for s in services
               if getattr(getattr(s, "config", None), "checkpoint", None) is not None and s.config.checkpoint.enabled]
    if not enabled:
        return
    policies = {s.name: s.config.checkpoint for s in enabled}
    if len(set(policies.values())) != 1:
        raise ValueError("every checkpointing service must share one GlobalCheckpointConfig (the resume point is an "
                         "intersection over shards), got: " + ", ".join(f"{k}={v}" for k, v in sorted(policies.items())))
    roles = {s.role for s in enabled}
    present = {s.role for s in services}
    for role in ("training", "critic", "rollout"):
        if role in present and role not in roles:
            raise ValueError(f"checkpointing is enabled but the {role!r} service does not carry the shared "
                             "GlobalCheckpointConfig; a resume would reset it")
    for c in [s for s in services if s.role == "critic"]:
        cold = int(getattr(c.config, "cold_start_windows", 0))
        for t in [s for s in services if s.role == "training"]:
            off = int(getattr(t.config, "critic_cold_start_windows", 0))
            if off != cold:
                raise ValueError(f"critic {c.name!r} cold_start_windows={cold} but trainer {t.name!r} "
                                 f"critic_cold_start_windows={off}; they number one gate stream and must match")


def _validate_critic_columns(services: list[ServiceInfo]) -> None:
    critics = [s for s in services if s.role == "critic"]
    trainers = [s for s in services if s.role == "training"]
    for c in critics:
        mode = getattr(c.config, "publish_mode", "advantage")
        published = set(CRITIC_OUTPUT_FIELDS_BY_MODE[mode])
        for t in trainers:
            fetched = set(getattr(t.config, "tq_fields", ()))
            if not published <= fetched:
                raise ValueError(f"critic {c.name!r} publishes {sorted(published)} (publish_mode={mode!r}) but trainer "
                                 f"{t.name!r} fetches {sorted(fetched)}; the trainer would never see a scored row")
            gae = bool(getattr(getattr(t.config, "trainer_params", None), "enable_gae", False))
            if mode == "values" and not gae:
                raise ValueError(f"critic {c.name!r} publishes per-token values but trainer {t.name!r} has "
                                 "enable_gae=False")
            if mode != "values" and gae:
                raise ValueError(f"trainer {t.name!r} has enable_gae=True but critic {c.name!r} does not publish values")


def _attach_colocations(services: list[ServiceInfo], rings: list) -> None:
    if not rings:
        return
    ids = [r.group_id for r in rings]
    if len(set(ids)) != len(ids):
        raise ValueError(f"duplicate colocation group ids: {ids}")
    known = {s.group_id for s in services}
    assigned: set[str] = set()
    for ring in rings:
        members = {n.service_id for n in ring.ring}
        if members - known:
            raise ValueError(f"colocation {ring.group_id!r} references unknown groups: {sorted(members - known)}")
        if members & assigned:
            raise ValueError(f"ServiceGroups can belong to only one colocation ring: {sorted(members & assigned)}")
        assigned |= members
        cards = {g: frozenset(x.global_rank for s in services if s.group_id == g for x in s.replica_gpus)
                 for g in members}
        if len(set(cards.values())) != 1:
            raise ValueError(f"colocation ring {ring.group_id!r} members do not share the same GPU block: "
                             f"{ {k: sorted(v) for k, v in cards.items()} }")
        for g in members:
            ms = [s for s in services if s.group_id == g]
            if not ms or not all(s.is_colocate for s in ms):
                raise ValueError(f"colocation ring member {g!r} is not placed on colocated GPUs")
            for s in ms:
                s.colocation = ring
                s.is_colocation_leader = s.replica_idx == 0


def _validate_ports(services: list[ServiceInfo]) -> None:
    for attr in ("endpoint_port", "dist_port"):
        owners: dict = {}
        for s in services:
            if not s.uses_gpu:
                continue
            port = getattr(s, attr)
            if not 1 <= port <= 65535:
                raise ValueError(f"service {s.name!r} has invalid {attr} {port}")
            key = (s.host, port)
            if key in owners:
                raise ValueError(f"{attr} collision on {s.host}:{port} between services {owners[key]!r} and "
                                 f"{s.name!r}; choose distinct port bases")
            owners[key] = s.name


__all__ = ["ServiceInfo", "Topology", "build_topology"]
