"""Run-level bootstrap key/value store (a ``torch.distributed.TCPStore``).

The launcher (or global rank 0) hosts it; everyone else connects through
``XRL_BOOTSTRAP_ADDR`` / ``XRL_BOOTSTRAP_PORT``.  It carries readiness markers
and the data-plane endpoint, so no shared filesystem is needed across nodes
(reference ``meshy/service/bootstrap.py``).  :func:`wait_keys` polls with a
liveness probe so a dead dependency fails the wait instead of hanging it.
"""

from __future__ import annotations

import os
import time
from datetime import timedelta
from typing import Callable, Sequence

ADDR_ENV, PORT_ENV, TIMEOUT_ENV = "XRL_BOOTSTRAP_ADDR", "XRL_BOOTSTRAP_PORT", "XRL_BOOTSTRAP_TIMEOUT"
_STORE = None


def _tcp_store(host: str, port: int, is_master: bool, timeout: float):
    from torch.distributed import TCPStore

    return TCPStore(host, port, world_size=None, is_master=is_master, timeout=timedelta(seconds=timeout),
                    wait_for_workers=False, use_libuv=True)


def host_store(host: str = "127.0.0.1", port: int = 0, timeout: float = 3600.0):
    """Host the store in this process and export its address to children."""
    global _STORE
    _STORE = _tcp_store(host, port, True, timeout)
    os.environ[ADDR_ENV] = host
    os.environ[PORT_ENV] = str(_STORE.port)
    return _STORE


def get_store(timeout: float | None = None):
    global _STORE
    if _STORE is not None:
        return _STORE
    host = os.environ.get(ADDR_ENV)
    port = os.environ.get(PORT_ENV)
    if not host or not port:
        raise RuntimeError(f"bootstrap store not configured ({ADDR_ENV}/{PORT_ENV} unset)")
    t = float(timeout if timeout is not None else os.environ.get(TIMEOUT_ENV, "3600"))
    _STORE = _tcp_store(host, int(port), False, t)
    return _STORE


def set_store(store) -> None:
    """Install a store object (tests use ``torch.distributed.HashStore``)."""
    global _STORE
    _STORE = store


def mark(key: str, value: str = "1") -> None:
    get_store().set(key, value)


def check(keys: Sequence[str]) -> bool:
    return bool(get_store().check(list(keys)))


def wait_keys(keys: Sequence[str], *, timeout: float = 1800.0, interval: float = 0.5,
              liveness: Callable[[], bool] | None = None) -> None:
    deadline = time.monotonic() + timeout
    keys = list(keys)
    while True:
        if check(keys):
            return
        if liveness is not None and not liveness():
            raise RuntimeError(f"a dependency died while waiting for {keys}")
        if time.monotonic() > deadline:
            raise TimeoutError(f"timed out after {timeout}s waiting for {keys}")
        time.sleep(interval)


__all__ = ["check", "get_store", "host_store", "mark", "set_store", "wait_keys"]
