"""Host-side fault injection: make chosen calls of a client, ledger or transport fail, vanish or stall.

The reference has no fault injection; it only detects failures (liveness-probed waits, bounded retries,
timeouts: ``meshy/worker/tq.py:257-276``, ``meshy/engine/sglang.py:96-121``, ``meshy/service/colocation.py:
252-277``). This module lets a test or an operator exercise those paths on purpose, always on the host: a
wrapped object's method raises a transport error, returns without doing anything (a message that is dropped),
or sleeps before doing its work (a slow peer). Nothing here touches a GPU.

A plan maps scopes to method rules; each rule is a list of actions taken by that method's successive calls,
after which the method behaves normally again::

    tq:get_data=raise*2,put=delay0.5; ledger:create=drop

* ``raise`` -- raise :class:`InjectedFault` (a ``ConnectionError``) instead of calling;
* ``drop`` -- return ``None`` without calling (a lost write);
* ``delay<seconds>`` -- sleep, then call;
* ``pass`` -- call normally (to skip some calls before a fault);
* ``<action>*<n>`` repeats an action ``n`` times.

:func:`inject` wraps an object when the plan (argument, or the ``XRL_FAULTS`` environment variable) has rules
for its scope and returns it unchanged otherwise, so the hooks cost nothing in a normal run. The column-store
client (:func:`meshy_b200.tq.client.connect`, scope ``tq``) and the colocation ledger of the inference service
(scope ``ledger``) pass through it.
"""

from __future__ import annotations

import os
import threading
import time
from typing import Any, Mapping, Sequence

ENV = "XRL_FAULTS"


class InjectedFault(ConnectionError):
    """The error a ``raise`` action throws."""


def _expand(actions: Sequence[str]) -> list[str]:
    out: list[str] = []
    for a in actions:
        a = a.strip()
        if not a:
            continue
        name, _, count = a.partition("*")
        n = int(count) if count else 1
        if n < 0:
            raise ValueError(f"negative repeat count in fault action {a!r}")
        if not (name in ("raise", "drop", "pass") or (name.startswith("delay") and _delay(name) >= 0)):
            raise ValueError(f"unknown fault action {a!r}")
        out += [name] * n
    return out


def _delay(name: str) -> float:
    try:
        return float(name[len("delay"):])
    except ValueError:
        raise ValueError(f"fault action {name!r}: 'delay' takes seconds, e.g. delay0.5") from None


def parse_plan(spec: str) -> dict[str, dict[str, list[str]]]:
    """``"scope:method=a,b,...; scope2:..."`` -> ``{scope: {method: [action, ...]}}``."""
    plan: dict[str, dict[str, list[str]]] = {}
    for part in spec.split(";"):
        part = part.strip()
        if not part:
            continue
        scope, sep, rules = part.partition(":")
        if not sep or not scope.strip():
            raise ValueError(f"fault plan entry {part!r} needs 'scope:method=actions'")
        methods = plan.setdefault(scope.strip(), {})
        # "m1=a,b,m2=c": an item with '=' starts a new method; the others continue the current one
        current = None
        for item in rules.split(","):
            if "=" in item:
                current, _, first = item.partition("=")
                current = current.strip()
                methods.setdefault(current, []).extend(_expand([first]))
            elif current is None:
                raise ValueError(f"fault plan entry {part!r}: action {item!r} before any 'method='")
            else:
                methods[current].extend(_expand([item]))
    return plan


class FaultyProxy:
    """Wraps ``target``: each call of a method with rules takes the next action of its list (thread-safe);
    everything else is the target's. ``events`` records ``(method, action)`` of every injected action."""

    def __init__(self, target: Any, rules: Mapping[str, Sequence[str]], scope: str = ""):
        self._target = target
        self._rules = {m: list(_expand(a)) for m, a in rules.items()}
        self._scope = scope
        self._lock = threading.Lock()
        self.events: list[tuple[str, str]] = []

    def _next(self, method: str) -> str | None:
        with self._lock:
            q = self._rules.get(method)
            if not q:
                return None
            action = q.pop(0)
            if action != "pass":
                self.events.append((method, action))
            return action

    def pending(self) -> int:
        """Actions not taken yet (0 once the plan has played out)."""
        with self._lock:
            return sum(len(q) for q in self._rules.values())

    def __getattr__(self, name: str) -> Any:
        attr = getattr(self._target, name)
        if name not in self._rules or not callable(attr):
            return attr

        def call(*args, **kwargs):
            action = self._next(name)
            if action == "raise":
                raise InjectedFault(f"injected fault: {self._scope or type(self._target).__name__}.{name}")
            if action == "drop":
                return None
            if action is not None and action.startswith("delay"):
                time.sleep(_delay(action))
            return attr(*args, **kwargs)

        return call


def inject(obj: Any, scope: str, plan: str | Mapping[str, Mapping[str, Sequence[str]]] | None = None) -> Any:
    """``obj`` wrapped in a :class:`FaultyProxy` if the plan has rules for ``scope``, else ``obj`` itself."""
    if plan is None:
        plan = os.environ.get(ENV, "")
    if isinstance(plan, str):
        if not plan.strip():
            return obj
        plan = parse_plan(plan)
    rules = plan.get(scope)
    return FaultyProxy(obj, rules, scope) if rules else obj


__all__ = ["ENV", "FaultyProxy", "InjectedFault", "inject", "parse_plan"]
