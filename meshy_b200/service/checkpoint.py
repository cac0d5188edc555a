"""Global checkpoints of a run: per-service shards with a commit protocol, and the resume point.

On-disk format (kept from the reference, ``meshy/service/checkpoint.py``, so
a run directory reads the same under both)::

    state/<service>/step-<n>/           the shard (a DCP directory or role files)
    state/<service>/step-<n>.json       sidecar {service, global_step, created_at, payload}
    state/<service>/step-<n>.complete   commit marker

Commit protocol: a writer fills the shard, writes the sidecar, and writes the
marker last; each file goes to a temporary name, is fsync'd and renamed, so a
crash leaves either a committed step or an uncommitted one, never a torn
marker. Removal inverts the order (marker first), so a half-removed step is
never mistaken for a committed one.

Resume point: the newest step that *every* service taking part at that step
committed. Each service commits on its own schedule, so this is an
intersection computed from one directory scan per service; nobody
coordinates at save time.
"""

from __future__ import annotations

import json
import os
import shutil
import time
from typing import Any, Callable, Iterable, Sequence

RESUME_ENV = "XRL_RESUME"
RESUME_STEP_ENV = "XRL_RESUME_STEP"

_MARK = ".complete"
_SIDECAR = ".json"
_PREFIX = "step-"


def resume_requested() -> bool:
    """``XRL_RESUME`` set to anything but empty / 0 / false / no."""
    return os.environ.get(RESUME_ENV, "").strip().lower() not in {"", "0", "false", "no"}


def run_resume_step() -> int:
    """The resume step the ignitor published for this run (0 = fresh start)."""
    raw = os.environ.get(RESUME_STEP_ENV) or "0"
    return int(raw)


def _durable_write(path: str, text: str) -> None:
    parent = os.path.dirname(path)
    os.makedirs(parent, exist_ok=True)
    staging = path + ".partial"
    fd = os.open(staging, os.O_WRONLY | os.O_CREAT | os.O_TRUNC, 0o644)
    try:
        os.write(fd, text.encode("utf-8"))
        os.fsync(fd)
    finally:
        os.close(fd)
    os.rename(staging, path)


def _step_of(entry: str, suffix: str) -> int | None:
    """``step-<n><suffix>`` -> n, anything else -> None."""
    if not (entry.startswith(_PREFIX) and entry.endswith(suffix)):
        return None
    digits = entry[len(_PREFIX):len(entry) - len(suffix)]
    return int(digits) if digits.isdigit() else None


class StateStore:
    """The ``state/`` directory of a run."""

    def __init__(self, state_dir: str):
        self.root = os.path.abspath(state_dir)

    # ------------------------------------------------------------------ paths
    def service_dir(self, service: str) -> str:
        return os.path.join(self.root, service)

    def _base(self, service: str, step: int) -> str:
        return os.path.join(self.service_dir(service), "%s%d" % (_PREFIX, int(step)))

    def shard_dir(self, service: str, step: int) -> str:
        return self._base(service, step)

    def meta_path(self, service: str, step: int) -> str:
        return self._base(service, step) + _SIDECAR

    def marker_path(self, service: str, step: int) -> str:
        return self._base(service, step) + _MARK

    # ------------------------------------------------------------------ commit
    def write_meta(self, service: str, step: int, payload: dict[str, Any]) -> str:
        path = self.meta_path(service, step)
        doc = {"created_at": time.time(), "global_step": int(step), "payload": payload, "service": service}
        _durable_write(path, json.dumps(doc, indent=2, sort_keys=True))
        return path

    def mark_complete(self, service: str, step: int) -> None:
        _durable_write(self.marker_path(service, step), str(int(step)))

    # ------------------------------------------------------------------ queries
    def read_meta(self, service: str, step: int) -> dict | None:
        try:
            with open(self.meta_path(service, step), encoding="utf-8") as f:
                return json.load(f)
        except (OSError, ValueError):
            return None

    def payload(self, service: str, step: int) -> dict:
        doc = self.read_meta(service, step) or {}
        return dict(doc.get("payload") or {})

    def _entries(self, path: str) -> list[str]:
        try:
            return os.listdir(path)
        except (FileNotFoundError, NotADirectoryError):
            return []

    def complete_steps(self, service: str) -> list[int]:
        found = (_step_of(e, _MARK) for e in self._entries(self.service_dir(service)))
        return sorted(s for s in found if s is not None)

    def is_complete(self, service: str, step: int) -> bool:
        return os.path.isfile(self.marker_path(service, step))

    def known_services(self) -> list[str]:
        return sorted(e for e in self._entries(self.root) if os.path.isdir(os.path.join(self.root, e)))

    def has_any_shard(self) -> bool:
        return any(self.complete_steps(svc) for svc in self.known_services())

    # ------------------------------------------------------------------ removal
    def drop(self, service: str, step: int) -> None:
        """Uncommit first (marker), then the sidecar and the shard."""
        for path in (self.marker_path(service, step), self.meta_path(service, step)):
            if os.path.lexists(path):
                os.remove(path)
        shutil.rmtree(self.shard_dir(service, step), ignore_errors=True)

    def prune(self, service: str, keep_latest_k: int) -> list[int]:
        """Drop all but the newest ``keep_latest_k`` committed steps of ``service`` (k <= 0 keeps all)."""
        if keep_latest_k <= 0:
            return []
        steps = self.complete_steps(service)
        old = steps[:max(0, len(steps) - keep_latest_k)]
        for s in old:
            self.drop(service, s)
        return old

    def drop_newer_than(self, step: int) -> dict[str, list[int]]:
        """Remove every service's commits past ``step`` (a resumed run rewrites them)."""
        removed: dict[str, list[int]] = {}
        for svc in self.known_services():
            newer = [s for s in self.complete_steps(svc) if s > step]
            for s in newer:
                self.drop(svc, s)
            if newer:
                removed[svc] = newer
        return removed


def resolve_resume_step(store: StateStore, participants_at: Callable[[int], Sequence[str]], *,
                        candidates: Iterable[int] | None = None) -> int:
    """Newest step at which every participant (``participants_at(step)``) committed; 0 if none."""
    committed = {svc: set(store.complete_steps(svc)) for svc in store.known_services()}
    pool = set(candidates) if candidates is not None else set().union(*committed.values()) if committed else set()
    for step in sorted(pool, reverse=True):
        who = list(participants_at(step))
        if who and all(step in committed.get(svc, ()) for svc in who):
            return int(step)
    return 0


__all__ = ["RESUME_ENV", "RESUME_STEP_ENV", "StateStore", "resolve_resume_step", "resume_requested",
           "run_resume_step"]
