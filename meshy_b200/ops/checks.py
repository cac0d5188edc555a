"""Index validation in front of the native kernels (debug mode: ``MESHY_CHECK_INDICES=1``).

The kernels trust their index inputs, for speed: token ids index the embedding and the LM head, slot
mappings and block tables index the paged KV cache, expert ids index the stacked expert weights. A wrong
index there reads or writes outside a buffer on the GPU instead of raising, and such a fault can leave the
device unusable. With the switch on, each entry point checks its indices before the launch and raises
``IndexError`` naming the op and the offending value. A check reads two scalars back to the host, so the
mode is for debugging only. Checks are skipped while a CUDA graph is being captured (a host read would
break the capture): run the workload eagerly once with the switch on to check what the graphs replay.
"""

from __future__ import annotations

import os

import torch

_ENABLED = os.environ.get("MESHY_CHECK_INDICES", "0") == "1"


def set_enabled(flag: bool) -> None:
    global _ENABLED
    _ENABLED = bool(flag)


def enabled() -> bool:
    if not _ENABLED:
        return False
    return not (torch.cuda.is_available() and torch.cuda.is_current_stream_capturing())


def check_range(what: str, t: torch.Tensor | None, lo: int, hi: int, *, skip_negative: bool = False) -> None:
    """Every entry of ``t`` in ``[lo, hi)`` (entries below zero exempt with ``skip_negative``: "no index")."""
    if not enabled() or t is None or t.numel() == 0:
        return
    v = t.reshape(-1)
    if skip_negative:
        v = v[v >= 0]
        if v.numel() == 0:
            return
    mn, mx = int(v.min()), int(v.max())
    if mn < lo or mx >= hi:
        bad = mn if mn < lo else mx
        raise IndexError(f"{what}: index {bad} outside [{lo}, {hi})")


def check_paged(what: str, block_table: torch.Tensor, seq_lens: torch.Tensor, n_pages: int, page: int) -> None:
    """Each row's length fits its block-table row, and the pages it uses are cache pages."""
    if not enabled() or block_table.numel() == 0:
        return
    max_pages = block_table.shape[1]
    check_range(f"{what} sequence lengths", seq_lens, 0, max_pages * page + 1)
    used = torch.arange(max_pages, device=block_table.device)[None, :] < \
        ((seq_lens.long() + page - 1) // page)[:, None]
    check_range(f"{what} block table", block_table[used], 0, n_pages)


__all__ = ["check_paged", "check_range", "enabled", "set_enabled"]
