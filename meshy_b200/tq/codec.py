"""Cell codec: one column value of one row <-> bytes.

Tensors travel as ``b"T" | dtype code | ndim | shape (int64) | raw bytes``;
anything else as ``b"P" | pickle``.  No pickling for tensors means no O(B^2)
object graphs and zero-copy decode with ``torch.frombuffer``.
"""

from __future__ import annotations

import pickle
import struct

import numpy as np
import torch

_DT = [torch.float32, torch.float64, torch.float16, torch.bfloat16, torch.int64, torch.int32, torch.int16,
       torch.int8, torch.uint8, torch.bool]
_CODE = {d: i for i, d in enumerate(_DT)}


def encode(value) -> bytes:
    if isinstance(value, torch.Tensor):
        t = value.detach()
        if t.is_cuda:
            t = t.cpu()
        t = t.contiguous()
        code = _CODE.get(t.dtype)
        if code is not None:
            hdr = struct.pack(f"<cBB{t.dim()}q", b"T", code, t.dim(), *t.shape)
            raw = t.view(torch.uint8).numpy().tobytes() if t.dtype == torch.bfloat16 else t.numpy().tobytes()
            return hdr + raw
    if isinstance(value, (int, float, bool)) and not isinstance(value, np.generic):
        return encode(torch.tensor(value))
    return b"P" + pickle.dumps(value, protocol=pickle.HIGHEST_PROTOCOL)


def decode(blob: bytes):
    if blob[:1] == b"P":
        return pickle.loads(blob[1:])
    code, ndim = struct.unpack_from("<BB", blob, 1)
    shape = struct.unpack_from(f"<{ndim}q", blob, 3)
    off = 3 + 8 * ndim
    dt = _DT[code]
    n = 1
    for s in shape:
        n *= s
    if n == 0:
        return torch.empty(shape, dtype=dt)
    buf = bytearray(blob[off:])
    if dt == torch.bfloat16:
        return torch.frombuffer(buf, dtype=torch.uint8).view(torch.bfloat16).reshape(shape)
    return torch.frombuffer(buf, dtype=dt).reshape(shape)


__all__ = ["decode", "encode"]
