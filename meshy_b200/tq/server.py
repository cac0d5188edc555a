"""TCP front end of the native column store (one process serves a whole run).

Replaces the reference's TransferQueue controller + storage units
(``meshy/transferqueue/launch.py:46-281``): the data and the AND-filter live
in the C++ :class:`meshy_b200._native.ColumnStore`; this module only frames
requests (msgpack, length-prefixed) over one thread per connection.  Blocking
``get_meta`` waits release the GIL inside the store.

    python -m meshy_b200.tq.server --host 127.0.0.1 --port 0 [--publish-key K]
"""

from __future__ import annotations

import argparse
import socket
import socketserver
import threading

from .client import _recv, _send

_OPS = {"put_rows", "put_columns", "get_meta", "get_data", "clear", "clear_partition", "reset_consumption",
        "partitions", "num_rows", "status"}


class _Handler(socketserver.BaseRequestHandler):
    def handle(self):
        store = self.server.store
        sock: socket.socket = self.request
        sock.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
        while True:
            try:
                op, args = _recv(sock)
            except (ConnectionError, OSError):
                return
            try:
                if op not in _OPS:
                    raise ValueError(f"unknown op {op!r}")
                result = getattr(store, op)(*args)
                if isinstance(result, list) and op == "status":
                    result = [list(x) for x in result]
                _send(sock, [True, result])
            except Exception as e:  # report to the client, keep serving
                _send(sock, [False, f"{type(e).__name__}: {e}"])


class ColumnStoreServer(socketserver.ThreadingTCPServer):
    daemon_threads = True
    allow_reuse_address = True

    def __init__(self, host: str = "127.0.0.1", port: int = 0, store=None):
        super().__init__((host, port), _Handler)
        if store is None:
            from .._native import ColumnStore

            store = ColumnStore()
        self.store = store

    @property
    def endpoint(self) -> str:
        host, port = self.server_address[:2]
        return f"{host}:{port}"

    def start_background(self) -> threading.Thread:
        t = threading.Thread(target=self.serve_forever, name="column-store", daemon=True)
        t.start()
        return t


def main(argv=None):
    p = argparse.ArgumentParser(description="meshy_b200 column store server")
    p.add_argument("--host", default="127.0.0.1")
    p.add_argument("--port", type=int, default=0)
    p.add_argument("--publish-key", default=None, help="write the endpoint under this bootstrap-store key")
    a = p.parse_args(argv)
    srv = ColumnStoreServer(a.host, a.port)
    print(f"column store listening on {srv.endpoint}", flush=True)
    if a.publish_key:
        from ..service.bootstrap import get_store

        get_store().set(a.publish_key, srv.endpoint)
    srv.serve_forever()


if __name__ == "__main__":
    main()
