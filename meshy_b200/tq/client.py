"""TransferQueue-shaped client API over the native column store.

Same surface the reference's workers use (``meshy/worker/tq.py:205-305``,
``meshy/transferqueue/control.py``): ``put(data, partition_id=...)`` appends
rows, ``put(data, metadata=meta)`` writes columns onto fetched rows,
``get_meta(data_fields, batch_size, partition_id, mode, task_name)`` returns a
:class:`BatchMeta` (AND-filter over produced columns, per-task consumption),
``get_data(meta)`` the values, ``clear_samples(meta)`` deletes rows.

``data`` is a :class:`Columns` batch (dict of column -> list of per-row
values, the role TensorDict plays upstream; jagged rows are simply lists of
differently sized tensors).  Two transports share the API: :class:`LocalClient`
calls the store in-process; :class:`RemoteClient` talks to
:mod:`meshy_b200.tq.server` over TCP.
"""

from __future__ import annotations

import socket
import struct
import threading
from dataclasses import dataclass, field
from typing import Any, Iterable, Mapping, Sequence

import msgpack

from .codec import decode, encode

_MODES = {"fetch": 0, "force_fetch": 1, "insert": 2}


class Columns(dict):
    """A batch of rows in column form: ``{field: [v_row0, v_row1, ...]}``."""

    @property
    def batch_size(self) -> tuple[int]:
        n = len(next(iter(self.values()))) if dict.__len__(self) else 0
        return (n,)

    def __len__(self) -> int:  # number of rows, like TensorDict's batch dim
        return self.batch_size[0]

    def keys(self):  # noqa: D401 - dict API
        return super().keys()

    def row(self, i: int) -> dict:
        return {k: v[i] for k, v in self.items()}

    @classmethod
    def from_rows(cls, rows: Sequence[Mapping[str, Any]], fields: Iterable[str] | None = None) -> "Columns":
        fields = list(fields) if fields is not None else (list(rows[0].keys()) if rows else [])
        return cls({f: [r[f] for r in rows] for f in fields})


@dataclass
class BatchMeta:
    partition_id: str
    global_indexes: list[int] = field(default_factory=list)
    fields: list[str] = field(default_factory=list)

    @property
    def size(self) -> int:
        return len(self.global_indexes)


class _Base:
    def put(self, data: Mapping[str, Sequence[Any]], partition_id: str | None = None,
            metadata: BatchMeta | None = None) -> BatchMeta:
        fields = list(data.keys())
        vals = [[encode(v) for v in data[f]] for f in fields]
        if metadata is not None:
            self._call("put_columns", metadata.partition_id, list(metadata.global_indexes), fields, vals)
            return BatchMeta(metadata.partition_id, list(metadata.global_indexes), fields)
        if partition_id is None:
            raise ValueError("put needs partition_id or metadata")
        idx = self._call("put_rows", partition_id, fields, vals)
        return BatchMeta(partition_id, list(idx), fields)

    def get_meta(self, data_fields: Sequence[str], batch_size: int, partition_id: str, mode: str = "fetch",
                 task_name: str = "default", wait_ms: int = 0) -> BatchMeta:
        if mode not in _MODES:
            raise ValueError(f"unknown get_meta mode {mode!r}")
        idx = self._call("get_meta", partition_id, list(data_fields), int(batch_size), _MODES[mode], task_name,
                         int(wait_ms))
        return BatchMeta(partition_id, list(idx), list(data_fields))

    def get_data(self, meta: BatchMeta, fields: Sequence[str] | None = None) -> Columns:
        fields = list(fields) if fields is not None else list(meta.fields)
        if meta.size == 0:
            return Columns({f: [] for f in fields})
        cols = self._call("get_data", meta.partition_id, list(meta.global_indexes), fields)
        return Columns({f: [decode(b) for b in col] for f, col in zip(fields, cols)})

    def clear_samples(self, meta: BatchMeta) -> int:
        return int(self._call("clear", meta.partition_id, list(meta.global_indexes)))

    def clear_partition(self, partition_id: str) -> None:
        self._call("clear_partition", partition_id)

    def reset_consumption(self, meta: BatchMeta, task_name: str) -> None:
        self._call("reset_consumption", meta.partition_id, task_name, list(meta.global_indexes))

    def num_rows(self, partition_id: str) -> int:
        return int(self._call("num_rows", partition_id))

    def production_status(self, partition_id: str, fields: Sequence[str]) -> list[tuple[int, int]]:
        return [tuple(x) for x in self._call("status", partition_id, list(fields))]

    def close(self) -> None:
        pass


class LocalClient(_Base):
    """In-process client (tests, single-process runs, the server itself)."""

    def __init__(self, store=None):
        if store is None:
            from .._native import ColumnStore

            store = ColumnStore()
        self.store = store

    def _call(self, op: str, *args):
        return getattr(self.store, op)(*args)


def _send(sock: socket.socket, obj) -> None:
    payload = msgpack.packb(obj, use_bin_type=True)
    sock.sendall(struct.pack("<Q", len(payload)) + payload)


def _recv_exact(sock: socket.socket, n: int) -> bytes:
    buf = bytearray(n)
    view = memoryview(buf)
    got = 0
    while got < n:
        k = sock.recv_into(view[got:], n - got)
        if k == 0:
            raise ConnectionError("column store connection closed")
        got += k
    return bytes(buf)


def _recv(sock: socket.socket):
    (n,) = struct.unpack("<Q", _recv_exact(sock, 8))
    return msgpack.unpackb(_recv_exact(sock, n), raw=False)


class RemoteClient(_Base):
    """TCP client of :mod:`meshy_b200.tq.server` (one connection, thread-safe)."""

    def __init__(self, endpoint: str, timeout: float = 60.0):
        host, port = endpoint.rsplit(":", 1)
        self.endpoint = endpoint
        self.sock = socket.create_connection((host, int(port)), timeout=timeout)
        self.sock.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
        self.lock = threading.Lock()

    def _call(self, op: str, *args):
        with self.lock:
            _send(self.sock, [op, list(args)])
            ok, result = _recv(self.sock)
        if not ok:
            raise RuntimeError(f"column store {op} failed: {result}")
        return result

    def close(self) -> None:
        try:
            self.sock.close()
        except OSError:
            pass


def connect(ref: str | None = None) -> _Base:
    """``tcp://host:port`` / ``host:port`` → RemoteClient; ``store://key`` reads the
    endpoint from the bootstrap store; ``None`` → a fresh in-process store. The client
    goes through :func:`meshy_b200.utils.faults.inject` (scope ``tq``), a no-op unless a
    fault plan names that scope."""
    from ..utils.faults import inject

    if ref is None or ref == "local":
        return inject(LocalClient(), "tq")
    if ref.startswith("store://"):
        from ..service.bootstrap import get_store

        key = ref[len("store://"):]
        endpoint = get_store().get(key).decode()
        return inject(RemoteClient(endpoint), "tq")
    if ref.startswith("tcp://"):
        ref = ref[len("tcp://"):]
    return inject(RemoteClient(ref), "tq")


__all__ = ["BatchMeta", "Columns", "LocalClient", "RemoteClient", "connect"]
