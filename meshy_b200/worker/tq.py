"""Data-plane driven role loop (reference ``meshy/worker/tq.py:19-383``).

A :class:`TQWorker` declares one primary input (AND-filter over ``fields`` in
``partition``, consumed as task ``consumer``), optional control inputs
(gates) and named outputs (new rows, or columns written back onto the input
rows).  ``run_tq_once``: fetch → read → ``process_tq_batch`` → write → clear,
each phase retried independently; a phase that keeps failing raises
:class:`TQWorkerError` to ``on_tq_fatal``.  Async helpers let an asyncio
producer (the rollout) share one client through a single-thread executor.
"""

from __future__ import annotations

import asyncio
import logging
import time
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass
from typing import Any, Callable, Mapping, Sequence

from ..tq.client import Columns, connect
from .base import Worker

log = logging.getLogger(__name__)


@dataclass(frozen=True)
class TQInput:
    partition: str
    fields: Sequence[str]
    batch_size: int
    consumer: str
    clear_after_success: bool = True

    def __post_init__(self) -> None:
        if not self.fields:
            raise ValueError("TQInput needs at least one field")
        if not self.consumer:
            raise ValueError("TQInput needs a consumer task name")


@dataclass(frozen=True)
class TQOutput:
    fields: Sequence[str]
    new_rows: bool = False
    partition: str | None = None

    def __post_init__(self) -> None:
        if self.new_rows and not self.partition:
            raise ValueError("a new-row TQOutput needs a partition")


class TQWorkerError(RuntimeError):
    pass


class TQWorker(Worker):
    tq_max_retries = 3
    tq_process_retries = 0
    tq_retry_interval = 1.0

    def __init__(self):
        super().__init__()
        self.tq_input: TQInput | None = None
        self.tq_controls: dict[str, TQInput] = {}
        self.tq_outputs: dict[str, TQOutput] = {}
        self.tq_poll_interval = 0.5
        self.tq_paused = None
        self._endpoints_ref: str | None = None
        self._client_factory: Callable[[], Any] | None = None
        self._tq_stats = {"consumed": 0, "produced": 0, "batches": 0, "errors": 0, "process_seconds": 0.0}
        self._exec: ThreadPoolExecutor | None = None
        self._aclient = None
        self.fatal: BaseException | None = None

    def configure_tq(self, *, endpoints_ref: str | None = None, input: TQInput | None = None,
                     controls: Mapping[str, TQInput] | None = None, outputs: Mapping[str, TQOutput] | None = None,
                     poll_interval: float = 0.5, client_factory: Callable[[], Any] | None = None) -> None:
        self._endpoints_ref = endpoints_ref
        self.tq_input = input
        self.tq_controls = dict(controls or {})
        self.tq_outputs = dict(outputs or {})
        self.tq_poll_interval = poll_interval
        self._client_factory = client_factory

    def _connect_tq(self):
        return self._client_factory() if self._client_factory else connect(self._endpoints_ref)

    # ------------------------------------------------------------------ hooks
    def process_tq_batch(self, samples: list[dict]) -> dict[str, Columns]:
        raise NotImplementedError

    def startup_tq_outputs(self) -> dict[str, Columns]:
        return {}

    def should_clear_batch(self) -> bool:
        return bool(self.tq_input and self.tq_input.clear_after_success)

    def on_tq_fatal(self, exc: BaseException) -> None:
        self.fatal = exc
        log.exception("%s fatal: %s", type(self).__name__, exc)

    # ------------------------------------------------------------------ loop
    def run(self) -> None:
        client = self._connect_tq()
        try:
            start = self.startup_tq_outputs()
            if start:
                self._retry("startup-write", lambda: self._write(client, None, start), self.tq_max_retries, 0)
            while not self.stopped:
                if self.tq_paused is not None and self.tq_paused.is_set():
                    self._worker_stop.wait(self.tq_poll_interval)
                    continue
                if not self.run_tq_once(client):
                    self._worker_stop.wait(self.tq_poll_interval)
        except BaseException as exc:  # noqa: BLE001
            self.on_tq_fatal(exc)
        finally:
            client.close()

    def run_tq_once(self, client) -> bool:
        if self.tq_input is None:
            raise RuntimeError("run_tq_once requires a primary TQ input")
        spec = self.tq_input
        try:
            meta = client.get_meta(data_fields=list(spec.fields), batch_size=spec.batch_size,
                                   partition_id=spec.partition, mode="fetch", task_name=spec.consumer)
        except Exception as e:
            self._tq_stats["errors"] += 1
            log.warning("get_meta failed: %s", e)
            return False
        if meta.size == 0:
            return False
        t0 = time.monotonic()
        data = self._retry("read", lambda: client.get_data(meta), self.tq_max_retries, meta.size)
        samples = [data.row(i) for i in range(meta.size)]
        result = self._retry("process", lambda: self.process_tq_batch(samples), self.tq_process_retries, meta.size)
        self._retry("write", lambda: self._write(client, meta, result), self.tq_max_retries, meta.size)
        if self.should_clear_batch():
            self._retry("clear", lambda: client.clear_samples(meta), self.tq_max_retries, meta.size)
        self._tq_stats["consumed"] += meta.size
        self._tq_stats["batches"] += 1
        self._tq_stats["process_seconds"] += time.monotonic() - t0
        return True

    def _retry(self, phase: str, fn: Callable[[], Any], retries: int, n: int) -> Any:
        last = None
        for attempt in range(retries + 1):
            try:
                return fn()
            except BaseException as e:  # noqa: BLE001
                last = e
                self._tq_stats["errors"] += 1
                if attempt >= retries:
                    break
                log.warning("%s %s phase failed for batch %d (attempt %d/%d): %s", type(self).__name__, phase, n,
                            attempt + 1, retries + 1, e)
                if self._worker_stop.wait(self.tq_retry_interval):
                    break
        raise TQWorkerError(f"{type(self).__name__} failed {phase} phase for batch of {n} after {retries + 1} "
                            "attempt(s)") from last

    def _write(self, client, meta, result: Mapping[str, Columns]) -> None:
        if not isinstance(result, Mapping):
            raise TypeError(f"process_tq_batch must return a mapping, got {type(result).__name__}")
        unknown = set(result) - set(self.tq_outputs)
        if unknown:
            raise ValueError(f"undeclared outputs: {sorted(unknown)}")
        for name, data in result.items():
            spec = self.tq_outputs[name]
            if set(data.keys()) != set(spec.fields):
                raise ValueError(f"output {name!r} fields mismatch: expected {sorted(spec.fields)}, "
                                 f"got {sorted(data.keys())}")
            if spec.new_rows:
                client.put(data=data, partition_id=spec.partition)
            else:
                if meta is None:
                    raise ValueError(f"output {name!r} cannot modify rows without input metadata")
                if len(data) != meta.size:
                    raise ValueError(f"output {name!r} has {len(data)} rows, input has {meta.size}")
                client.put(data=data, metadata=meta)
            self._tq_stats["produced"] += len(data)

    # ------------------------------------------------------------------ async side
    async def open_tq(self) -> None:
        self._exec = ThreadPoolExecutor(max_workers=1, thread_name_prefix="tq-client")
        self._aclient = await asyncio.get_running_loop().run_in_executor(self._exec, self._connect_tq)

    async def tq_call(self, fn: Callable[..., Any], *args) -> Any:
        return await asyncio.get_running_loop().run_in_executor(self._exec, fn, *args)

    async def write_tq_output(self, name: str, data: Columns) -> None:
        if name not in self.tq_outputs:
            raise ValueError(f"output {name!r} is not declared")
        await self.tq_call(lambda: self._retry("write", lambda: self._write(self._aclient, None, {name: data}),
                                               self.tq_max_retries, len(data)))
        self._tq_stats["batches"] += 1

    async def read_tq_control(self, name: str) -> Columns | None:
        spec = self.tq_controls[name]

        def read():
            meta = self._aclient.get_meta(data_fields=list(spec.fields), batch_size=spec.batch_size,
                                          partition_id=spec.partition, mode="fetch", task_name=spec.consumer)
            if meta.size == 0:
                return None
            d = self._aclient.get_data(meta)
            if spec.clear_after_success:
                self._aclient.clear_samples(meta)
            return d

        return await self.tq_call(read)

    async def close_tq(self) -> None:
        if self._exec is None:
            return
        if self._aclient is not None:
            await asyncio.get_running_loop().run_in_executor(self._exec, self._aclient.close)
        self._exec.shutdown(wait=True)
        self._exec = None
        self._aclient = None

    def health_info(self) -> dict[str, Any]:
        info = super().health_info()
        info.update({f"tq/{k}": v for k, v in self._tq_stats.items()})
        return info


__all__ = ["TQInput", "TQOutput", "TQWorker", "TQWorkerError"]
