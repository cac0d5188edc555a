"""Decentralised GPU ownership for colocated services: a token ring over a request ledger.

Every service of a ring (e.g. inference FALLBACK, trainer ON_DEMAND) owns a
:class:`ColocationManager`.  Ownership moves only by *grants* written into a
shared ledger, one row per request:

* a service that needs the card posts a request (``request_gpu``) and waits
  for a grant naming that request;
* the current owner, on ``release`` (or, if it is a FALLBACK owner, as soon as
  any open request appears: preemption), picks the next owner among open
  requests by ``(priority, ring distance from the owner, age)`` — ON_DEMAND
  requests (priority 0) beat FALLBACK ones (priority 1) — calls its
  ``on_release`` callback (free memory *before* publishing), closes its own
  request and writes the grant;
* grants carry a contiguous sequence number; a manager applying a grant that
  skips a number or whose source is not the previous target raises (the
  ledger is corrupt), and the genesis grant (sequence 0) must name the ring's
  first member;
* a FALLBACK member that lost the card keeps a standing FALLBACK request so
  the token can always return to it; an ON_DEMAND owner that releases with no
  other requester waits ``next_owner_timeout`` for the next ring member, then
  hands the card back to the fallback owner.

The protocol is the reference's (``meshy/service/colocation.py:24-518``)
because all members must agree on it; the code is this package's.  Ledgers:
:class:`MemoryLedger` (one process, tests) and :class:`StoreLedger` (rows of
a column-store partition, for services in different processes).
"""

from __future__ import annotations

import logging
import queue
import threading
import time
import uuid
from concurrent.futures import Future
from concurrent.futures import TimeoutError as FutureTimeout
from contextlib import contextmanager
from dataclasses import dataclass, replace
from enum import Enum
from typing import Any, Callable, Iterator, NamedTuple, Protocol

log = logging.getLogger(__name__)


class SchedulingMode(str, Enum):
    ON_DEMAND = "on_demand"
    FALLBACK = "fallback"


RequestKind = SchedulingMode


class RingNode(NamedTuple):
    service_id: str
    mode: SchedulingMode


@dataclass(frozen=True)
class ColocationRing:
    """Members of one card block in hand-off order; ``ring[0]`` holds the card first."""

    group_id: str
    ring: tuple
    poll_interval: float = 1.0
    next_owner_timeout: float = 3.0

    def __post_init__(self) -> None:
        nodes = tuple(RingNode(str(sid), SchedulingMode(mode)) for sid, mode in self.ring)
        object.__setattr__(self, "ring", nodes)
        object.__setattr__(self, "_index", {n.service_id: i for i, n in enumerate(nodes)})
        problems = []
        if not self.group_id:
            problems.append("group_id is empty")
        if len(nodes) < 2:
            problems.append(f"{len(nodes)} member(s); a hand-off needs two or more")
        if any(not n.service_id for n in nodes):
            problems.append("a member has an empty service id")
        if len(self._index) != len(nodes):
            problems.append("a service appears twice: " + ", ".join(n.service_id for n in nodes))
        if not self.poll_interval > 0:
            problems.append(f"poll_interval {self.poll_interval} is not positive")
        if self.next_owner_timeout < 0:
            problems.append(f"next_owner_timeout {self.next_owner_timeout} is negative")
        if problems:
            raise ValueError(f"colocation ring {self.group_id!r}: " + "; ".join(problems))

    @property
    def initial_owner(self) -> str:
        return self.ring[0].service_id

    def ring_index_for(self, service_id: str) -> int:
        try:
            return self._index[service_id]
        except KeyError:
            raise KeyError(f"{service_id!r} is not a member of colocation ring {self.group_id!r}") from None

    def mode_for(self, service_id: str) -> SchedulingMode:
        return self.ring[self.ring_index_for(service_id)].mode


@dataclass(frozen=True)
class GpuRequest:
    group_id: str
    service_id: str
    request_id: str
    created_at_ns: int
    payload_ref: str | None = None
    ring_index: int = 0
    priority: int = 0
    kind: SchedulingMode = SchedulingMode.ON_DEMAND


@dataclass(frozen=True)
class GpuGrant:
    group_id: str
    sequence: int
    source: str
    target: str
    request_id: str | None = None
    transition: str = ""
    payload_ref: str | None = None


@dataclass
class LedgerRow:
    request: GpuRequest
    state: str = "open"           # open | granted | closed
    grant: GpuGrant | None = None


class Ledger(Protocol):
    def create(self, request: GpuRequest) -> None: ...
    def grant(self, request_id: str, grant: GpuGrant) -> None: ...
    def close(self, request_id: str) -> None: ...
    def scan(self) -> list[LedgerRow]: ...
    def shutdown(self) -> None: ...


class MemoryLedger:
    """Ledger shared by managers living in one process (tests, single-process runs)."""

    def __init__(self):
        self._rows: dict[str, LedgerRow] = {}
        self._lock = threading.Lock()

    def create(self, request: GpuRequest) -> None:
        with self._lock:
            self._rows[request.request_id] = LedgerRow(request)

    def grant(self, request_id: str, grant: GpuGrant) -> None:
        with self._lock:
            row = self._rows[request_id]
            row.state, row.grant = "granted", grant

    def close(self, request_id: str) -> None:
        with self._lock:
            if request_id in self._rows:
                self._rows[request_id].state = "closed"

    def scan(self) -> list[LedgerRow]:
        with self._lock:
            return [LedgerRow(r.request, r.state, r.grant) for r in self._rows.values()]

    def shutdown(self) -> None:
        pass


class StoreLedger:
    """Ledger rows in a column-store partition ``control.colocate.<group>.request``."""

    FIELDS = ["request", "state", "grant"]

    def __init__(self, client, group_id: str):
        self.client = client
        self.partition = f"control.colocate.{group_id}.request"

    def _rows(self):
        meta = self.client.get_meta(self.FIELDS, 0, self.partition, mode="force_fetch")
        if meta.size == 0:
            return meta, {}
        return meta, self.client.get_data(meta)

    def _find(self, request_id: str):
        meta, data = self._rows()
        if not data:
            raise KeyError(request_id)
        for i, req in enumerate(data["request"]):
            if req["request_id"] == request_id:
                from ..tq.client import BatchMeta

                return BatchMeta(self.partition, [meta.global_indexes[i]], self.FIELDS)
        raise KeyError(request_id)

    def create(self, request: GpuRequest) -> None:
        from ..tq.client import Columns

        req = dict(request.__dict__)
        req["kind"] = request.kind.value
        self.client.put(Columns({"request": [req], "state": ["open"], "grant": [None]}), partition_id=self.partition)

    def grant(self, request_id: str, grant: GpuGrant) -> None:
        from ..tq.client import Columns

        self.client.put(Columns({"state": ["granted"], "grant": [dict(grant.__dict__)]}),
                        metadata=self._find(request_id))

    def close(self, request_id: str) -> None:
        from ..tq.client import Columns

        try:
            self.client.put(Columns({"state": ["closed"]}), metadata=self._find(request_id))
        except KeyError:
            pass

    def scan(self) -> list[LedgerRow]:
        _, data = self._rows()
        out = []
        for req, state, grant in zip(data.get("request", []), data.get("state", []), data.get("grant", [])):
            r = GpuRequest(**{**req, "kind": SchedulingMode(req["kind"])})
            out.append(LedgerRow(r, state, GpuGrant(**grant) if grant else None))
        return out

    def shutdown(self) -> None:
        pass


GENESIS_SOURCE = "authority"


def issue_genesis(config: ColocationRing, ledger: Ledger) -> GpuGrant:
    """Write the ring's first grant (sequence 0, from the authority to ``ring[0]``) into an empty ledger."""
    owner = config.initial_owner
    request = GpuRequest(group_id=config.group_id, service_id=owner, request_id="genesis:" + config.group_id,
                         created_at_ns=0, ring_index=0, priority=1, kind=SchedulingMode.FALLBACK)
    grant = GpuGrant(group_id=config.group_id, sequence=0, source=GENESIS_SOURCE, target=owner,
                     request_id=request.request_id, transition="genesis")
    ledger.create(request)
    ledger.grant(request.request_id, grant)
    return grant


class _Command(NamedTuple):
    """Work handed to the manager thread; the caller waits on ``future``."""

    action: str
    payload: Any
    future: Future


class ColocationManager:
    """One service's view of the ring; a background thread reconciles the ledger."""

    def __init__(self, config: ColocationRing, service_id: str, ledger_factory: Callable[[], Ledger], *,
                 on_acquire: Callable[[GpuGrant], None] | None = None,
                 on_release: Callable[[str], None] | None = None, command_timeout: float = 30.0):
        config.ring_index_for(service_id)
        self.config = config
        self.service_id = service_id
        self.mode = config.mode_for(service_id)
        self._ledger_factory = ledger_factory
        self._on_acquire = on_acquire or (lambda g: None)
        self._on_release = on_release or (lambda target: None)
        self._cmds: queue.Queue[_Command] = queue.Queue()
        self._stop = threading.Event()
        self._started = threading.Event()
        self._thread: threading.Thread | None = None
        self._fatal: BaseException | None = None
        self._rows: dict[str, LedgerRow] = {}
        self._grants: dict[str, GpuGrant] = {}
        self._events: dict[str, threading.Event] = {}
        self._acquired: set[int] = set()
        self._owner: str | None = None
        self._last_seq = -1
        self._grant: GpuGrant | None = None
        self._transferring = False
        self.command_timeout = command_timeout

    # ------------------------------------------------------------------ public
    @property
    def owns_gpu(self) -> bool:
        return self._owner == self.service_id

    @property
    def owner(self) -> str | None:
        return self._owner

    @property
    def fatal_error(self) -> BaseException | None:
        return self._fatal

    def start(self) -> None:
        if self._thread is not None:
            raise RuntimeError("ColocationManager is already started")
        self._thread = threading.Thread(target=self._run, daemon=True,
                                        name=f"colocate-{self.config.group_id}-{self.service_id}")
        self._thread.start()
        if not self._started.wait(30):
            raise TimeoutError(f"colocation manager {self.service_id} did not start")

    def request_gpu(self, request_id: str | None = None, payload_ref: str | None = None, *,
                    kind: SchedulingMode | None = None) -> GpuRequest:
        kind = kind or SchedulingMode.ON_DEMAND
        req = GpuRequest(self.config.group_id, self.service_id, request_id or uuid.uuid4().hex, time.time_ns(),
                         payload_ref, self.config.ring_index_for(self.service_id),
                         0 if kind is SchedulingMode.ON_DEMAND else 1, kind)
        self._submit("request", req)
        return req

    def wait_for_grant(self, request: GpuRequest, timeout: float | None = None) -> GpuGrant:
        ev = self._events.setdefault(request.request_id, threading.Event())
        if not ev.wait(timeout):
            raise TimeoutError(f"timed out waiting for request {request.request_id!r}")
        if self._fatal is not None:
            raise RuntimeError("colocation manager failed") from self._fatal
        return self._grants[request.request_id]

    @contextmanager
    def occupy(self, request: GpuRequest, *, transition: str = "") -> Iterator[GpuGrant]:
        g = self.wait_for_grant(request)
        try:
            yield g
        finally:
            self.release(transition=transition)

    def release(self, *, transition: str = "", payload_ref: str | None = None):
        return self._submit("release", (transition, payload_ref))

    def stop(self) -> None:
        if self._thread is None:
            return
        if self._thread.is_alive():
            try:
                self._submit("stop", None)
            except Exception:
                self._stop.set()
            self._thread.join(timeout=10)
        self._thread = None

    # ------------------------------------------------------------------ loop
    def _submit(self, action: str, payload: Any):
        if self._thread is None:
            raise RuntimeError("ColocationManager is not started")
        if self._fatal is not None:
            raise RuntimeError("colocation manager failed") from self._fatal
        fut: Future = Future()
        self._cmds.put(_Command(action, payload, fut))
        try:
            return fut.result(timeout=self.command_timeout)
        except FutureTimeout:
            raise TimeoutError(f"colocation command {action!r} timed out") from None

    def _run(self) -> None:
        ledger = self._ledger_factory()
        try:
            self._started.set()
            while not self._stop.is_set():
                self._drain(ledger)
                self._reconcile(ledger.scan(), ledger)
                self._stop.wait(self.config.poll_interval)
        except BaseException as exc:  # noqa: BLE001 - surfaced to every waiter
            self._fatal = exc
            log.exception("colocation manager %s failed", self.service_id)
            while True:
                try:
                    pending = self._cmds.get_nowait()
                except queue.Empty:
                    break
                pending.future.set_exception(exc)
            for ev in self._events.values():
                ev.set()
        finally:
            ledger.shutdown()

    def _drain(self, ledger: Ledger) -> None:
        while True:
            try:
                cmd = self._cmds.get_nowait()
            except queue.Empty:
                return
            try:
                if cmd.action == "request":
                    ledger.create(cmd.payload)
                    self._rows[cmd.payload.request_id] = LedgerRow(cmd.payload)
                    result = cmd.payload
                elif cmd.action == "release":
                    self._reconcile(ledger.scan(), ledger)
                    result = self._transfer(ledger, *cmd.payload)
                elif cmd.action == "stop":
                    self._stop.set()
                    result = None
                else:
                    raise ValueError(f"unknown colocation command {cmd.action!r}")
            except BaseException as e:  # noqa: BLE001 - handed to the waiting caller
                cmd.future.set_exception(e)
            else:
                cmd.future.set_result(result)

    def _reconcile(self, rows: list[LedgerRow], ledger: Ledger) -> None:
        rows.sort(key=lambda r: r.grant.sequence if r.grant else -1)
        for row in rows:
            rid = row.request.request_id
            prev = self._rows.get(rid)
            self._rows[rid] = row
            if row.state == "open" and row.grant is None and row.request.service_id != self.service_id \
                    and self.owns_gpu and self.mode is SchedulingMode.FALLBACK and not self._transferring:
                self._transfer(ledger, "preempt", None)
                continue
            if row.grant is None:
                continue
            if prev is not None and prev.grant is not None and prev.grant.sequence >= row.grant.sequence:
                continue
            self._apply(row.grant)
            if self.mode is SchedulingMode.FALLBACK and not self.owns_gpu:
                self._ensure_fallback(ledger)

    def _ensure_fallback(self, ledger: Ledger, service_id: str | None = None) -> None:
        sid = service_id or self.service_id
        for r in self._rows.values():
            q = r.request
            if q.service_id == sid and q.kind is SchedulingMode.FALLBACK and r.state == "open" and r.grant is None:
                return
        req = GpuRequest(self.config.group_id, sid, f"{sid}:fallback:{self._last_seq + 1}", time.time_ns(),
                         ring_index=self.config.ring_index_for(sid), priority=1, kind=SchedulingMode.FALLBACK)
        ledger.create(req)
        self._rows[req.request_id] = LedgerRow(req)

    def _apply(self, g: GpuGrant) -> None:
        if g.group_id != self.config.group_id or g.sequence <= self._last_seq:
            return
        if self._last_seq < 0:
            if g.sequence != 0 or g.source != GENESIS_SOURCE or g.target != self.config.initial_owner:
                raise RuntimeError(f"invalid genesis grant: {g}")
        elif g.sequence != self._last_seq + 1 or self._grant is None or g.source != self._grant.target:
            raise RuntimeError(f"non-contiguous GPU grant: last={self._grant}, next={g}")
        self._last_seq = g.sequence
        self._grant = g
        self._owner = g.target
        if g.request_id:
            self._grants[g.request_id] = g
        if g.target == self.service_id and g.sequence not in self._acquired:
            self._acquired.add(g.sequence)
            self._on_acquire(g)
        if g.request_id:
            self._events.setdefault(g.request_id, threading.Event()).set()

    def _candidates(self):
        me = self.config.ring_index_for(self.service_id)
        n = len(self.config.ring)
        out = []
        for r in self._rows.values():
            q = r.request
            if r.state != "open" or r.grant is not None or q.group_id != self.config.group_id \
                    or q.service_id == self.service_id:
                continue
            out.append((q.priority, (q.ring_index - me) % n, q.created_at_ns, q.request_id, r))
        out.sort(key=lambda c: c[:4])
        return out

    def _select_next(self, ledger: Ledger) -> LedgerRow | None:
        if not self.owns_gpu:
            return None
        c = self._candidates()
        if c:
            return c[0][4]
        if self._grant is not None and self._grant.source not in (self.service_id, GENESIS_SOURCE):
            # nobody asked: hand the card back to whoever gave it to us
            self._ensure_fallback(ledger, self._grant.source)
            c = self._candidates()
            return c[0][4] if c else None
        return None

    def _transfer(self, ledger: Ledger, transition: str, payload_ref: str | None):
        if not self.owns_gpu:
            raise RuntimeError(f"service {self.service_id!r} does not own the GPU")
        if self._transferring:
            raise RuntimeError(f"colocation {self.config.group_id}: transfer re-entered on {self.service_id!r}")
        self._transferring = True
        try:
            nxt = self.config.ring[(self.config.ring_index_for(self.service_id) + 1) % len(self.config.ring)]
            deadline = time.monotonic() + self.config.next_owner_timeout
            while time.monotonic() < deadline and not any(
                    r.request.service_id == nxt.service_id and r.state == "open" and r.grant is None
                    for r in self._rows.values()):
                time.sleep(min(0.05, self.config.poll_interval))
                for row in ledger.scan():
                    self._rows.setdefault(row.request.request_id, row)
                    if row.state != self._rows[row.request.request_id].state:
                        self._rows[row.request.request_id] = row
            sel = self._select_next(ledger)
            if sel is None:
                log.warning("colocation %s: nobody requested the GPU; keeping it", self.config.group_id)
                return None
            target = sel.request.service_id
            self._on_release(target)
            if self._grant is not None and self._grant.request_id:
                ledger.close(self._grant.request_id)
                if self._grant.request_id in self._rows:
                    self._rows[self._grant.request_id].state = "closed"
            g = GpuGrant(self.config.group_id, self._last_seq + 1, self.service_id, target, sel.request.request_id,
                         transition, payload_ref)
            ledger.grant(sel.request.request_id, g)
            sel.state, sel.grant = "granted", g
            self._apply(g)
            log.info("colocation transfer %s -> %s (seq=%d, %s)", g.source, g.target, g.sequence, transition)
            return g
        finally:
            self._transferring = False


class NoopColocationManager:
    owns_gpu = True

    def start(self) -> None: ...

    def request_gpu(self, request_id=None, payload_ref=None, **kw) -> GpuRequest:
        return GpuRequest("", "", request_id or uuid.uuid4().hex, time.time_ns(), payload_ref)

    def wait_for_grant(self, request, timeout=None) -> GpuGrant:
        return GpuGrant("", 0, "", "", request.request_id)

    @contextmanager
    def occupy(self, request, **kw):
        yield self.wait_for_grant(request)

    def release(self, **kw) -> None: ...

    def stop(self) -> None: ...


__all__ = ["ColocationManager", "ColocationRing", "GpuGrant", "GpuRequest", "Ledger", "LedgerRow", "MemoryLedger",
           "NoopColocationManager", "RequestKind", "RingNode", "SchedulingMode", "StoreLedger", "issue_genesis"]
