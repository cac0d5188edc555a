"""Worker thread lifecycle (reference ``meshy/worker/base.py:9-58``)."""

from __future__ import annotations

import threading
from typing import Any


class Worker:
    def __init__(self):
        self._worker_stop = threading.Event()
        self._thread: threading.Thread | None = None

    @property
    def stopped(self) -> bool:
        return self._worker_stop.is_set()

    def run(self) -> None:
        raise NotImplementedError

    def start(self) -> threading.Thread:
        if self._thread is not None:
            raise RuntimeError("worker already started")
        self._thread = threading.Thread(target=self.run, name=type(self).__name__, daemon=True)
        self._thread.start()
        return self._thread

    def stop(self, timeout: float | None = 10.0) -> None:
        self._worker_stop.set()
        if self._thread is not None and self._thread is not threading.current_thread():
            self._thread.join(timeout)

    def health_info(self) -> dict[str, Any]:
        return {"worker": type(self).__name__, "stopped": self.stopped,
                "alive": self._thread.is_alive() if self._thread else False}


__all__ = ["Worker"]
