"""Global checkpoint shards and resume-point derivation.

Layout per service: ``state/{svc}/step-N/`` (the shard: DCP directory or role
files), ``step-N.json`` (sidecar: counters, weight version ...) and
``step-N.complete`` (commit marker, written last, fsync'd and renamed into
place).  The resume point is the newest step at which every participant
committed — an intersection, so nobody has to coordinate (reference
``meshy/service/checkpoint.py:1-246``).
"""

from __future__ import annotations

import json
import os
import re
import shutil
import time
from typing import Any, Callable, Iterable, Sequence

RESUME_ENV = "XRL_RESUME"
RESUME_STEP_ENV = "XRL_RESUME_STEP"
_COMPLETE_RE = re.compile(r"^step-(\d+)\.complete$")


def resume_requested() -> bool:
    return os.environ.get(RESUME_ENV, "").strip().lower() not in ("", "0", "false", "no")


def _atomic_write(path: str, text: str) -> None:
    os.makedirs(os.path.dirname(path), exist_ok=True)
    tmp = f"{path}.tmp"
    with open(tmp, "w", encoding="utf-8") as f:
        f.write(text)
        f.flush()
        os.fsync(f.fileno())
    os.replace(tmp, path)


class StateStore:
    def __init__(self, state_dir: str):
        self.root = os.path.abspath(state_dir)

    def service_dir(self, service: str) -> str:
        return os.path.join(self.root, service)

    def shard_dir(self, service: str, step: int) -> str:
        return os.path.join(self.service_dir(service), f"step-{int(step)}")

    def meta_path(self, service: str, step: int) -> str:
        return os.path.join(self.service_dir(service), f"step-{int(step)}.json")

    def _complete_path(self, service: str, step: int) -> str:
        return os.path.join(self.service_dir(service), f"step-{int(step)}.complete")

    def write_meta(self, service: str, step: int, payload: dict[str, Any]) -> str:
        doc = {"service": service, "global_step": int(step), "created_at": time.time(), "payload": payload}
        path = self.meta_path(service, step)
        _atomic_write(path, json.dumps(doc, indent=2, sort_keys=True))
        return path

    def mark_complete(self, service: str, step: int) -> None:
        _atomic_write(self._complete_path(service, step), str(int(step)))

    def read_meta(self, service: str, step: int) -> dict | None:
        try:
            with open(self.meta_path(service, step), encoding="utf-8") as f:
                return json.load(f)
        except (FileNotFoundError, NotADirectoryError, json.JSONDecodeError):
            return None

    def payload(self, service: str, step: int) -> dict:
        return dict((self.read_meta(service, step) or {}).get("payload") or {})

    def complete_steps(self, service: str) -> list[int]:
        try:
            entries = os.listdir(self.service_dir(service))
        except (FileNotFoundError, NotADirectoryError):
            return []
        return sorted(int(m.group(1)) for m in map(_COMPLETE_RE.match, entries) if m)

    def is_complete(self, service: str, step: int) -> bool:
        return os.path.exists(self._complete_path(service, step))

    def known_services(self) -> list[str]:
        try:
            return sorted(n for n in os.listdir(self.root) if os.path.isdir(os.path.join(self.root, n)))
        except (FileNotFoundError, NotADirectoryError):
            return []

    def has_any_shard(self) -> bool:
        return any(self.complete_steps(s) for s in self.known_services())

    def prune(self, service: str, keep_latest_k: int) -> list[int]:
        if keep_latest_k <= 0:
            return []
        stale = self.complete_steps(service)[:-keep_latest_k]
        for s in stale:
            self.drop(service, s)
        return stale

    def drop_newer_than(self, step: int) -> dict[str, list[int]]:
        dropped = {}
        for svc in self.known_services():
            stale = [s for s in self.complete_steps(svc) if s > step]
            for s in stale:
                self.drop(svc, s)
            if stale:
                dropped[svc] = stale
        return dropped

    def drop(self, service: str, step: int) -> None:
        for p in (self._complete_path(service, step), self.meta_path(service, step)):
            try:
                os.remove(p)
            except FileNotFoundError:
                pass
        shutil.rmtree(self.shard_dir(service, step), ignore_errors=True)


def resolve_resume_step(store: StateStore, participants_at: Callable[[int], Sequence[str]], *,
                        candidates: Iterable[int] | None = None) -> int:
    """Newest step every participant completed; 0 when none (fresh start)."""
    if candidates is None:
        seen: set[int] = set()
        for svc in store.known_services():
            seen.update(store.complete_steps(svc))
        candidates = seen
    for step in sorted(candidates, reverse=True):
        who = participants_at(step)
        if who and all(store.is_complete(s, step) for s in who):
            return int(step)
    return 0


def run_resume_step() -> int:
    """The resume step the ignitor published for this run (0 = fresh)."""
    return int(os.environ.get(RESUME_STEP_ENV, "0") or 0)


__all__ = ["RESUME_ENV", "RESUME_STEP_ENV", "StateStore", "resolve_resume_step", "resume_requested", "run_resume_step"]
