"""Trainer → rollout-engine weight synchronisation.

Trainer and engines lay parameters out identically in one flat buffer
(:func:`meshy_b200.backend.flat.flatten_module`), so a sync never re-keys or
re-shapes anything. Three routes, fastest first:

* same process (:class:`~meshy_b200.rl.ColocatedGRPO`): one device copy of
  the trainer's bf16 compute weights into the engine's bf16 buffer;
* same node, other processes (the launcher's services, any DP size): every
  trainer rank keeps a bf16 snapshot of its weights in the engines' layout
  (:class:`DevicePublisher`; one device copy per publish) and exports a CUDA
  IPC handle of it. Rank 0 gathers the handles, keyed by GPU UUID, into one
  ``ipc-set:`` reference (:func:`encode_handle_set`) that travels through the
  colocation ring as ``payload_ref``. Each engine server maps the handle of
  the trainer rank on its own GPU (:func:`pick_handle`) and copies the
  snapshot into its weight buffer: one device-to-device copy, no disk. DDP
  ranks hold identical weights, so any rank's snapshot is a full replica;
* disk: HF safetensors export + ``/update_weights_from_disk`` (the checkpoint
  format, and what the reference does for every sync,
  ``meshy/engine/titan.py:80-123`` / ``meshy/engine/sglang.py:289-300``).

The reference has no device route; it gathers the full state dict to rank 0
and writes safetensors every step.
"""

from __future__ import annotations

import base64
import json
import pickle

import torch


def export_ipc_flat(flat: torch.Tensor) -> str:
    """Serialise a CUDA tensor as an IPC handle string (same node only)."""
    from torch.multiprocessing.reductions import reduce_tensor

    if not flat.is_cuda:
        raise ValueError("IPC export needs a CUDA tensor")
    return base64.b64encode(pickle.dumps(reduce_tensor(flat))).decode()


def open_ipc_flat(handle: str, uuid: str | None = None) -> torch.Tensor:
    """Map an exported tensor. The handle names the exporter's device by ITS ordinal, which means nothing in a
    process with another ``CUDA_VISIBLE_DEVICES``; with ``uuid`` (the exporting GPU) the tensor is opened on
    this process's ordinal of that GPU."""
    fn, args = pickle.loads(base64.b64decode(handle.encode()))
    if uuid is not None:
        import inspect

        names = list(inspect.signature(fn).parameters)
        if "storage_device" in names:
            ordinal = local_ordinal(uuid)
            if ordinal is None:
                raise ValueError(f"GPU {uuid} is not visible in this process; cannot map its weights")
            args = list(args)
            args[names.index("storage_device")] = ordinal
    return fn(*args)


def local_ordinal(uuid: str) -> int | None:
    """This process's device ordinal of the GPU with ``uuid`` (None when it is not visible)."""
    for i in range(torch.cuda.device_count()):
        if device_uuid(i) == uuid:
            return i
    return None


def device_uuid(device: torch.device | int | None = None) -> str:
    """Stable identity of a GPU across processes (CUDA_VISIBLE_DEVICES renumbers ordinals, UUIDs stay)."""
    return str(torch.cuda.get_device_properties(device if device is not None else torch.cuda.current_device()).uuid)


class DevicePublisher:
    """One trainer rank's published weights: two bf16 snapshots used alternately.

    ``publish(version)`` copies the trainer's compute weights (bf16; the fp32
    master is cast when there is no bf16 copy) into the snapshot of
    ``version % 2`` and returns ``(gpu_uuid, version, handle)``. Two buffers let
    an engine still copying version ``v`` overlap the trainer publishing
    ``v + 1``. The snapshots stay on the GPU while the trainer is offloaded
    (2 bytes per parameter each)."""

    def __init__(self, flat, device):
        self.flat = flat
        self.device = torch.device(device)
        self.uuid = device_uuid(self.device)
        self._bufs: list[torch.Tensor | None] = [None, None]
        self._handles: list[str | None] = [None, None]

    def publish(self, version: int) -> tuple[str, int, str]:
        i = version % 2
        if self._bufs[i] is None:
            # the engines' (full) layout: a sharded trainer's own buffers hold only its shards
            n = getattr(self.flat, "global_numel", self.flat.numel)
            self._bufs[i] = torch.empty(n, dtype=torch.bfloat16, device=self.device)
            self._handles[i] = export_ipc_flat(self._bufs[i])
        src = self.flat.sync_source
        from ..ops.functional import native

        if src.dtype == self._bufs[i].dtype:
            self._bufs[i].copy_(src)
        elif native(src):
            from ..ops._ext import ext

            ext().cast_copy(src, self._bufs[i])
        else:
            self._bufs[i].copy_(src)
        torch.cuda.current_stream(self.device).synchronize()  # the snapshot is complete before it is announced
        return self.uuid, int(version), self._handles[i]


def encode_handle_set(entries) -> str:
    """``[(gpu_uuid, version, handle), ...]`` of every trainer rank → one ``ipc-set:`` reference."""
    versions = {int(v) for _, v, _ in entries}
    if len(versions) != 1:
        raise ValueError(f"trainer ranks published different weight versions: {sorted(versions)}")
    doc = {"version": versions.pop(), "handles": {u: h for u, _, h in entries}}
    return "ipc-set:" + json.dumps(doc, separators=(",", ":"))


def decode_handle_set(ref: str) -> dict:
    if not ref.startswith("ipc-set:"):
        raise ValueError("not an ipc-set reference")
    return json.loads(ref[len("ipc-set:"):])


def pick_handle(handles: dict[str, str], my_uuid: str) -> tuple[str, bool, str]:
    """The handle exported on this engine's GPU if there is one (``local=True``), else a visible peer GPU's
    (read over NVLink; any DDP rank's snapshot holds the same weights). Returns ``(handle, local, uuid)``."""
    if my_uuid in handles:
        return handles[my_uuid], True, my_uuid
    if not handles:
        raise ValueError("empty handle set")
    visible = [u for u in sorted(handles) if local_ordinal(u) is not None]
    u = visible[0] if visible else sorted(handles)[0]
    return handles[u], False, u


__all__ = ["DevicePublisher", "decode_handle_set", "device_uuid", "encode_handle_set", "export_ipc_flat",
           "local_ordinal", "open_ipc_flat", "pick_handle"]
