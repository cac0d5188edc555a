"""Clients of rollout engines (the reference's ``SGLangEngine``, ``meshy/engine/sglang.py``).

:class:`EngineClient` round-robins ``/generate`` over endpoints with retry +
linear backoff, and implements the abort/continuation loop: when a colocated
trainer preempts the engine, a request comes back with ``finish_reason=abort``
and its partial output; the client resubmits prompt + partial with the
remaining ``max_new_tokens`` and counts the continuation (the sample is then
stamped ``mixed_version``).  Non-finite log-probs are rejected.  Management
calls (pause/continue, release/resume memory, weight loads) fan out to every
endpoint.  :class:`LocalEngineClient` offers the same interface over an
in-process engine (single-process runs, tests).
"""

from __future__ import annotations

import asyncio
import itertools
import logging
import math
import threading
import time
from dataclasses import dataclass, field
from typing import Any, Iterable

log = logging.getLogger(__name__)


@dataclass
class Generation:
    output_ids: list = field(default_factory=list)
    output_logprobs: list = field(default_factory=list)
    finish_reason: str | None = None
    continuations: int = 0
    weight_version: int = -1

    def __iter__(self):  # unpacks as (tokens, logprobs)
        yield self.output_ids
        yield self.output_logprobs

    @property
    def truncated(self) -> bool:
        return self.finish_reason == "length"


class _Base:
    max_continuations = 128
    sampling_params: dict = {}

    async def _generate_once(self, prompt: list[int], params: dict) -> tuple[list, list, str, int]:
        raise NotImplementedError

    async def generate(self, input_ids: Iterable[int], sampling_params: dict | None = None) -> Generation:
        prompt = list(input_ids)
        params = dict(self.sampling_params if sampling_params is None else sampling_params)
        res = Generation()
        budget = params.get("max_new_tokens")
        for cont in range(self.max_continuations + 1):
            p = dict(params)
            if budget is not None:
                remaining = int(budget) - len(res.output_ids)
                if remaining <= 0:
                    res.finish_reason = "length"
                    return res
                p["max_new_tokens"] = remaining
            toks, lps, reason, version = await self._generate_once(prompt + res.output_ids, p)
            if any(not math.isfinite(x) for x in lps):
                raise ValueError("engine returned non-finite log-probs")
            res.output_ids.extend(toks)
            res.output_logprobs.extend(lps)
            res.weight_version = version
            if reason in ("stop", "length"):
                res.finish_reason = reason
                return res
            res.continuations += 1
        raise RuntimeError(f"generation did not finish after {self.max_continuations + 1} requests")


class EngineClient(_Base):
    def __init__(self, endpoints, sampling_params: dict | None = None, *, attempts: int = 60, backoff: float = 1.0,
                 backoff_max: float = 5.0, max_connections: int = 1024):
        if isinstance(endpoints, str):
            endpoints = [endpoints]
        self.endpoints = [e.rstrip("/") for e in endpoints]
        if not self.endpoints:
            raise ValueError("EngineClient requires at least one endpoint")
        self._cycle = itertools.cycle(self.endpoints)
        self._lock = threading.Lock()
        self.sampling_params = dict(sampling_params or {})
        self.attempts, self.backoff, self.backoff_max = max(1, attempts), backoff, backoff_max
        self.max_connections = max_connections
        self._session = None
        self.model_path: str | None = None

    def _next(self) -> str:
        with self._lock:
            return next(self._cycle)

    async def _sess(self):
        if self._session is None:
            import aiohttp

            self._session = aiohttp.ClientSession(connector=aiohttp.TCPConnector(limit=self.max_connections),
                                                  timeout=aiohttp.ClientTimeout(total=None, connect=30))
        return self._session

    async def _generate_once(self, prompt, params):
        url = f"{self._next()}/generate"
        payload = {"input_ids": prompt, "sampling_params": params, "return_logprob": True}
        last = None
        for i in range(self.attempts):
            try:
                s = await self._sess()
                async with s.post(url, json=payload) as r:
                    if r.status != 200:
                        raise RuntimeError(f"status {r.status}")
                    body = await r.json()
                meta = body.get("meta_info", {})
                lps = [x[0] for x in meta.get("output_token_logprobs", [])]
                reason = (meta.get("finish_reason") or {}).get("type")
                return list(body.get("output_ids", [])), lps, reason, int(meta.get("weight_version", -1))
            except Exception as e:  # transport failures are retryable
                last = e
                if i + 1 < self.attempts:
                    await asyncio.sleep(min(self.backoff * (i + 1), self.backoff_max))
        raise last

    # ------------------------------------------------------------------ management
    def _mgmt(self, method: str, path: str, timeout: float = 600.0, **kw) -> list:
        import requests

        out, last = [], None
        for ep in self.endpoints:
            try:
                r = getattr(requests, method.lower())(f"{ep}{path}", timeout=timeout, **kw)
                r.raise_for_status()
                out.append(r.json() if r.content else None)
            except requests.RequestException as e:
                last = e
        if last is not None:
            raise last
        return out

    def wait_ready(self, *, liveness=None, timeout: float = 1800.0) -> None:
        import requests

        deadline = time.monotonic() + timeout
        while time.monotonic() < deadline:
            if liveness is not None:
                liveness()
            try:
                if all(requests.get(f"{e}/health_generate", timeout=30).status_code == 200 for e in self.endpoints):
                    return
            except requests.RequestException:
                pass
            time.sleep(1.0)
        raise TimeoutError(f"engines not ready within {timeout}s: {self.endpoints}")

    def wait_until_idle(self, timeout: float = 300.0, interval: float = 0.2) -> None:
        deadline = time.monotonic() + timeout
        while time.monotonic() < deadline:
            loads = [l for r in self._mgmt("GET", "/v1/loads") for l in (r or {}).get("loads", [])]
            if sum(int(l.get("num_running_reqs", 0)) + int(l.get("num_waiting_reqs", 0)) for l in loads) == 0:
                return
            time.sleep(interval)
        raise TimeoutError("engines did not become idle")

    def pause_generation(self) -> None:
        self._mgmt("POST", "/pause_generation", json={"mode": "abort"})

    def weight_versions(self) -> list:
        """The weight version each endpoint serves."""
        return [(d or {}).get("weight_version") for d in self._mgmt("GET", "/get_model_info", timeout=30.0)]

    def continue_generation(self) -> None:
        self._mgmt("POST", "/continue_generation", json={})

    def release_memory(self, tags=("kv_cache", "weights")) -> None:
        self._mgmt("POST", "/release_memory_occupation", json={"tags": list(tags)})

    def resume_memory(self, tags=("kv_cache", "weights")) -> None:
        self._mgmt("POST", "/resume_memory_occupation", json={"tags": list(tags)})

    def load_weights(self, model_path: str, version: int | None = None) -> None:
        self._mgmt("POST", "/update_weights_from_disk", json={"model_path": model_path, "weight_version": version},
                   timeout=1800.0)

    def load_weights_ipc(self, handle: str, version: int | None = None) -> None:
        self._mgmt("POST", "/update_weights_from_ipc", json={"handle": handle, "weight_version": version},
                   timeout=1800.0)

    def load_weights_ipc_set(self, ref: str) -> None:
        """Every engine maps the trainer snapshot exported on its own GPU (``ipc-set:`` reference)."""
        from ..rollout.weight_sync import decode_handle_set

        doc = decode_handle_set(ref)
        self._mgmt("POST", "/update_weights_from_ipc", json={"handles": doc["handles"],
                                                              "weight_version": doc["version"]}, timeout=1800.0)

    def release_for_colocate(self) -> None:
        self.pause_generation()
        self.wait_until_idle()
        self.release_memory(("kv_cache", "weights"))

    def restore_for_colocate(self, payload_ref: str | None) -> None:
        self.resume_memory(("weights",))
        if payload_ref:
            if payload_ref.startswith("ipc-set:"):
                self.load_weights_ipc_set(payload_ref)
            elif payload_ref.startswith("ipc:"):
                self.load_weights_ipc(payload_ref[4:])
            else:
                self.load_weights(payload_ref)
        self.resume_memory(("kv_cache",))
        self.continue_generation()

    def on_colocate_release(self, target: str) -> None:
        self.release_for_colocate()

    def on_colocate_acquire(self, grant: Any) -> None:
        ref = getattr(grant, "payload_ref", None)
        if not ref and int(getattr(grant, "sequence", 0)) == 0:
            ref = self.model_path
        self.restore_for_colocate(ref)

    async def close(self) -> None:
        if self._session is not None:
            await self._session.close()
            self._session = None


class LocalEngineClient(_Base):
    """Same interface over an in-process :class:`~meshy_b200.rollout.RolloutEngine`."""

    def __init__(self, engine, sampling_params: dict | None = None):
        from ..rollout.server import EngineRunner

        self.runner = EngineRunner(engine)
        self.engine = engine
        self.sampling_params = dict(sampling_params or {})

    async def _generate_once(self, prompt, params):
        g = await self.runner.generate(prompt, params)
        return g.output_ids, g.output_logprobs, g.finish_reason, g.weight_version

    def pause_generation(self) -> None:
        self.runner.pause("abort")

    def weight_versions(self) -> list:
        return [self.engine.weight_version]

    def continue_generation(self) -> None:
        self.runner.resume()

    def close_sync(self) -> None:
        self.runner.shutdown()

    async def close(self) -> None:
        self.runner.shutdown()


__all__ = ["EngineClient", "Generation", "LocalEngineClient"]
