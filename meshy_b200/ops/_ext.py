"""Loader for the in-tree native extension ``meshy_b200._C``.

The extension holds every sm_100a kernel of the framework.  On a CUDA tensor
an op must run its kernel: if the extension is missing there, :func:`ext`
raises instead of silently computing the same thing with PyTorch ops.
"""

from __future__ import annotations

import importlib

_EXT = None
_ERR: Exception | None = None


def _load():
    global _EXT, _ERR
    if _EXT is not None or _ERR is not None:
        return _EXT
    try:
        _EXT = importlib.import_module("meshy_b200._C")
    except Exception as e:  # pragma: no cover - depends on the build
        _ERR = e
    return _EXT


def available() -> bool:
    return _load() is not None


def ext():
    mod = _load()
    if mod is None:
        raise RuntimeError(
            "meshy_b200._C (the sm_100a kernel library) is not built or failed to load: "
            f"{_ERR!r}. Build it with `python setup.py build_ext --inplace`."
        )
    return mod
