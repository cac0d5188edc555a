"""Trainer → rollout-engine weight synchronisation paths.

Both sides lay parameters out identically in one flat buffer
(:func:`meshy_b200.backend.flat.flatten_module`), so a sync never re-keys or
re-shapes anything:

* same process (colocated :class:`~meshy_b200.rl.ColocatedGRPO`): one cast
  kernel from the fp32 master buffer into the engine's bf16 buffer, or the
  AdamW kernel writes the engine buffer directly (``FlatAdamW.mirror``);
* same node, different process: the trainer exports its buffer as a CUDA IPC
  handle (:func:`export_ipc_flat`); the engine maps it (:func:`open_ipc_flat`)
  and copies device-to-device;
* different node / resharding (FSDP shards → full replicas): the NVLink
  reshard kernel in :mod:`meshy_b200.parallel.reshard`;
* disk: HF safetensors export + ``/update_weights_from_disk`` (checkpoint
  format, and the fallback the reference uses for every sync).
"""

from __future__ import annotations

import base64
import pickle

import torch


def export_ipc_flat(flat: torch.Tensor) -> str:
    """Serialise a CUDA tensor as an IPC handle string (same node only)."""
    from torch.multiprocessing.reductions import reduce_tensor

    if not flat.is_cuda:
        raise ValueError("IPC export needs a CUDA tensor")
    return base64.b64encode(pickle.dumps(reduce_tensor(flat))).decode()


def open_ipc_flat(handle: str) -> torch.Tensor:
    fn, args = pickle.loads(base64.b64decode(handle.encode()))
    return fn(*args)


__all__ = ["export_ipc_flat", "open_ipc_flat"]
