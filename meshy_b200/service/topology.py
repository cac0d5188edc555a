"""Service placement: a pure function from (recipe service groups, all GPUs of the job) to services.

Every rank evaluates :func:`build_topology` on the same inputs and so agrees
on the placement without talking to the others. The rules are the
reference's contract (``meshy/service/topology.py``), since recipes written
for it must land on the same cards and ports:

* GPU groups take consecutive blocks of cards in declaration order; a group
  with ``colocate_with=X`` takes X's block again (and must be the same size);
* replica ``r`` of a group owns the ``r``-th ``n_gpus_per_replica`` cards of
  its block; its ports are the config class's port bases plus the global rank
  of its first card (plus ``XRL_PORT_OFFSET``, default 0, which lets two runs
  share a host);
* CPU groups get no cards and no ports.

Then colocation rings are attached to their member services, and the whole
placement is checked (ports, ring membership, critic-to-trainer columns,
checkpoint policy) before any process starts; every problem found is
reported at once.
"""

from __future__ import annotations

import os
from dataclasses import dataclass, field
from typing import Any, Callable

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
        return rank in {g.global_rank for g in self.replica_gpus}

    @property
    def checkpoint_policy(self):
        ck = getattr(self.config, "checkpoint", None)
        return ck if ck is not None and ck.enabled else None


@dataclass
class Topology:
    services: list[ServiceInfo]

    def _where(self, pred: Callable[[ServiceInfo], bool]) -> list[ServiceInfo]:
        return [s for s in self.services if pred(s)]

    def group(self, gid: str) -> list[ServiceInfo]:
        return self._where(lambda s: s.group_id == gid)

    def by_name(self, name: str) -> ServiceInfo:
        hit = self._where(lambda s: s.name == name)
        if not hit:
            raise KeyError(f"topology has no service {name!r}")
        return hit[0]

    def gpu_services(self):
        return self._where(lambda s: s.uses_gpu)

    def cpu_services(self):
        return self._where(lambda s: not s.uses_gpu)

    def services_by_role(self, role: str):
        return self._where(lambda s: s.role == role)

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
        trainers = self.training_services()
        return trainers[0].endpoint if trainers else None

    def checkpointing_services(self):
        return self._where(lambda s: s.checkpoint_policy is not None)

    def checkpoint_config(self):
        ck = self.checkpointing_services()
        return ck[0].checkpoint_policy if ck else None

    def cold_start_windows(self) -> int:
        critics = self.services_by_role("critic")
        return int(getattr(critics[0].config, "cold_start_windows", 0)) if critics else 0

    def checkpoint_participants(self, step: int) -> tuple[str, ...]:
        """Services whose shard a resume at ``step`` needs. The trainer has none while the critic cold-starts
        (windows ``1..cold_start_windows``; a negative count means it never stops)."""
        cold = self.cold_start_windows()
        trainer_idle = cold < 0 or int(step) <= cold
        return tuple(s.name for s in self.checkpointing_services() if not (s.role == "training" and trainer_idle))

    def dependency_names(self, s: ServiceInfo) -> list[str]:
        return [dep.name for gid in s.wait_until for dep in self.group(gid)]

    def local_services(self, rank: int) -> list[ServiceInfo]:
        return [s for s in self.gpu_services() if s.contains_rank(rank)]

    def colocated_inference_for(self, trainer: ServiceInfo):
        """Inference replicas sharing the trainer's cards: names, {rank: name}, endpoints."""
        if trainer.colocate_with is None:
            return [], {}, []
        mine = {g.global_rank for g in trainer.replica_gpus}
        names, by_rank, endpoints = [], {}, []
        for inf in self.group(trainer.colocate_with):
            shared = [g.global_rank for g in inf.replica_gpus if g.global_rank in mine]
            if shared:
                names.append(inf.name)
                endpoints.append(inf.endpoint)
                by_rank.update({r: inf.name for r in shared})
        return names, by_rank, endpoints


def _port_offset() -> int:
    return int(os.environ.get("XRL_PORT_OFFSET", "0") or 0)


class _CardBlocks:
    """Hands out consecutive card blocks and remembers each group's block for its colocated followers."""

    def __init__(self, gpus: list[GPU]):
        self.free = sorted(gpus, key=lambda g: g.global_rank)
        self.next = 0
        self.of_group: dict[str, list[GPU]] = {}

    def block_for(self, sg: ServiceGroup) -> list[GPU]:
        want = sg.n_replicas * sg.n_gpus_per_replica
        if sg.colocate_with is not None:
            host = self.of_group.get(sg.colocate_with)
            if host is None:
                raise ValueError(f"{sg.id!r} colocates with {sg.colocate_with!r}, which is not a GPU group declared "
                                 "before it")
            if len(host) != want:
                raise ValueError(f"{sg.id!r} needs {want} cards but its colocation target {sg.colocate_with!r} "
                                 f"holds {len(host)}; colocated groups must be the same size")
            return host
        block = self.free[self.next:self.next + want]
        if len(block) < want:
            raise ValueError(f"{sg.id!r} needs {want} cards; only {len(block)} are left")
        self.next += want
        self.of_group[sg.id] = block
        return block


def build_topology(service_groups: list[ServiceGroup], gpus: list[GPU], colocations: list | None = None) -> Topology:
    cards = _CardBlocks(gpus)
    hosts_of_colocation = {sg.colocate_with for sg in service_groups if sg.colocate_with}
    offset = _port_offset()
    services: list[ServiceInfo] = []
    for sg in service_groups:
        cfg_type = type(sg.config)
        if not sg.role or sg.role == "?":
            raise ValueError(f"{cfg_type.__name__} declares no role")
        waits = list(sg.wait_until)
        if not sg.uses_gpu:
            services += [ServiceInfo(f"{sg.id}-{r}", sg.id, sg.role, False, r, "127.0.0.1", 0, 0, [], False, None,
                                     list(waits), sg.config) for r in range(sg.n_replicas)]
            continue
        if cfg_type.endpoint_port_base is None or cfg_type.dist_port_base is None:
            raise ValueError(f"{cfg_type.__name__} runs on GPUs, so it must declare endpoint_port_base and "
                             "dist_port_base")
        block = cards.block_for(sg)
        shared = sg.colocate_with is not None or sg.id in hosts_of_colocation
        per = sg.n_gpus_per_replica
        for r in range(sg.n_replicas):
            own = list(block[r * per:(r + 1) * per])
            first = own[0].global_rank
            services.append(ServiceInfo(
                f"{sg.id}-{r}", sg.id, sg.role, True, r, own[0].host, cfg_type.endpoint_port_base + first + offset,
                cfg_type.dist_port_base + first + offset, own, shared, sg.colocate_with, list(waits), sg.config))
    _attach_rings(services, colocations or [])
    problems = [p for check in (_port_problems, _critic_column_problems, _checkpoint_problems)
                for p in check(services)]
    if problems:
        raise ValueError("invalid service topology:\n  " + "\n  ".join(problems))
    return Topology(services)


def _attach_rings(services: list[ServiceInfo], rings: list) -> None:
    """Give each member service its ring (replica 0 of a group leads); rings must be disjoint and cover
    exactly one shared card block."""
    seen_ids: set[str] = set()
    taken: set[str] = set()
    groups = {s.group_id for s in services}
    for ring in rings:
        if ring.group_id in seen_ids:
            raise ValueError(f"colocation id {ring.group_id!r} is used twice")
        seen_ids.add(ring.group_id)
        members = {m.service_id for m in ring.ring}
        if not members <= groups:
            raise ValueError(f"colocation {ring.group_id!r} names groups that do not exist: {sorted(members - groups)}")
        if members & taken:
            raise ValueError(f"groups {sorted(members & taken)} appear in more than one colocation ring")
        taken |= members
        blocks = {g: frozenset(c.global_rank for s in services if s.group_id == g for c in s.replica_gpus)
                  for g in members}
        if len(set(blocks.values())) > 1:
            raise ValueError(f"members of colocation {ring.group_id!r} sit on different cards: "
                             f"{ {g: sorted(b) for g, b in blocks.items()} }")
        for g in members:
            mine = [s for s in services if s.group_id == g]
            if not mine or any(not s.is_colocate for s in mine):
                raise ValueError(f"{g!r} is in colocation {ring.group_id!r} but is not placed on shared cards")
            for s in mine:
                s.colocation, s.is_colocation_leader = ring, s.replica_idx == 0


def _port_problems(services: list[ServiceInfo]) -> list[str]:
    out = []
    for kind in ("endpoint_port", "dist_port"):
        claimed: dict[tuple[str, int], str] = {}
        for s in (x for x in services if x.uses_gpu):
            port = getattr(s, kind)
            if not 0 < port < 65536:
                out.append(f"{s.name}: {kind} {port} is outside 1..65535")
                continue
            other = claimed.setdefault((s.host, port), s.name)
            if other != s.name:
                out.append(f"{kind} collision: {other} and {s.name} both want {s.host}:{port} (give their configs "
                           "different port bases)")
    return out


def _critic_column_problems(services: list[ServiceInfo]) -> list[str]:
    out = []
    trainers = [s for s in services if s.role == "training"]
    for critic in (s for s in services if s.role == "critic"):
        mode = getattr(critic.config, "publish_mode", "advantage")
        produced = set(CRITIC_OUTPUT_FIELDS_BY_MODE[mode])
        for t in trainers:
            consumed = set(getattr(t.config, "tq_fields", ()))
            if not produced <= consumed:
                out.append(f"{t.name} never reads the critic's columns {sorted(produced - consumed)} "
                           f"(critic {critic.name}, publish_mode {mode!r})")
            wants_values = bool(getattr(getattr(t.config, "trainer_params", None), "enable_gae", False))
            if wants_values != (mode == "values"):
                out.append(f"{t.name} has enable_gae={wants_values} but critic {critic.name} publishes "
                           f"{'values' if mode == 'values' else 'advantages'}; GAE needs per-token values")
    return out


def _checkpoint_problems(services: list[ServiceInfo]) -> list[str]:
    on = [s for s in services if s.checkpoint_policy is not None]
    if not on:
        return []
    out = []
    if len({s.checkpoint_policy for s in on}) > 1:
        out.append("checkpointing services disagree on the GlobalCheckpointConfig (the resume point is the "
                   "newest step all of them saved): " + ", ".join(f"{s.name}={s.checkpoint_policy}" for s in on))
    missing = {s.role for s in services} - {s.role for s in on}
    for role in sorted(missing & {"training", "critic", "rollout"}):
        out.append(f"checkpointing is on but the {role} service has it off; a resume would restart that service "
                   "from scratch")
    for critic in (s for s in services if s.role == "critic"):
        cold = int(getattr(critic.config, "cold_start_windows", 0))
        for t in (s for s in services if s.role == "training"):
            if int(getattr(t.config, "critic_cold_start_windows", 0)) != cold:
                out.append(f"{t.name} critic_cold_start_windows differs from {critic.name} cold_start_windows "
                           f"({cold}); both count windows of one gate stream")
    return out


__all__ = ["ServiceInfo", "Topology", "build_topology"]
