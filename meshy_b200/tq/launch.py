"""Column-store (data plane) deployment: spec derivation and the server process.

Counterpart of the reference's TransferQueue cluster launcher and spec
(``meshy/transferqueue/launch.py:46-281``, ``meshy/transferqueue/spec.py:
30-57``).  The data plane here is one native column-store server (C++ store,
``meshy_b200._native``) instead of a controller plus storage units, so the
cluster is one subprocess; its endpoint goes to the bootstrap store under
``ENDPOINT_KEY`` and to ``XRL_TQ_ENDPOINTS`` for every child.

Sizing (``pre_alloc_sample_num``): the data partition must hold every sample
in flight at once -- batches the trainer has not consumed yet plus rollouts
still generating -- so ``max(4 * batch, 2 * max_running + batch, 1024)``.
"""

from __future__ import annotations

import os
import subprocess
import sys
import time
from typing import Any

ENDPOINT_KEY = "xrl/tq_endpoint"
_MIN_PRE_ALLOC = 1024


def derive_spec(service_groups, runtime_dir: str) -> dict[str, Any]:
    from ..config import RolloutServiceConfig, TrainingServiceConfig

    batch = 0
    running = 0
    for g in service_groups:
        if isinstance(g.config, TrainingServiceConfig):
            batch = max(batch, int(g.config.batch_size))
        elif isinstance(g.config, RolloutServiceConfig):
            running = max(running, int(g.config.async_max_running_request))
    pre = max(4 * batch, 2 * running + batch, _MIN_PRE_ALLOC)
    return {
        "endpoint": os.environ.get("XRL_TQ_ENDPOINTS"),
        "pre_alloc_sample_num": int(os.environ.get("XRL_TQ_PRE_ALLOC", str(pre))),
        "host": os.environ.get("XRL_TQ_HOST", "127.0.0.1"),
        "log": os.path.join(runtime_dir, "logs", "tq-server.log"),
    }


class ColumnStoreCluster:
    """Starts the column-store server subprocess and publishes its endpoint."""

    def __init__(self, spec: dict[str, Any]):
        self.spec = dict(spec)
        self.proc: subprocess.Popen | None = None
        self.endpoint: str | None = spec.get("endpoint")

    def start(self, timeout: float = 120.0) -> str:
        if self.endpoint:  # an external store was given
            os.environ["XRL_TQ_ENDPOINTS"] = self.endpoint
            return self.endpoint
        from ..service import bootstrap

        os.makedirs(os.path.dirname(self.spec["log"]), exist_ok=True)
        log = open(self.spec["log"], "ab")
        cmd = [sys.executable, "-m", "meshy_b200.tq.server", "--host", self.spec["host"], "--port", "0",
               "--publish-key", ENDPOINT_KEY]
        from ..service.base import die_with_parent

        self.proc = subprocess.Popen(cmd, stdout=log, stderr=subprocess.STDOUT, env=dict(os.environ),
                                     preexec_fn=die_with_parent)
        store = bootstrap.get_store()
        deadline = time.monotonic() + timeout
        while not store.check([ENDPOINT_KEY]):
            if self.proc.poll() is not None:
                raise RuntimeError(f"column store exited with code {self.proc.returncode}; see {self.spec['log']}")
            if time.monotonic() > deadline:
                raise TimeoutError("column store did not publish its endpoint")
            time.sleep(0.1)
        self.endpoint = store.get(ENDPOINT_KEY).decode()
        os.environ["XRL_TQ_ENDPOINTS"] = self.endpoint
        return self.endpoint

    def stop(self) -> None:
        if self.proc is not None and self.proc.poll() is None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=10)
            except subprocess.TimeoutExpired:
                self.proc.kill()


__all__ = ["ColumnStoreCluster", "ENDPOINT_KEY", "derive_spec"]
