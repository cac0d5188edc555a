"""Response-quality stamps (reference ``meshy/utils/metric.py:18-39``)."""

from __future__ import annotations

import zlib

REPETITION_MIN_CHARS = 10_000
REPETITION_COMPRESSION_RATIO = 10.0


def compression_ratio(text: str) -> float:
    raw = text.encode("utf-8", errors="replace")
    if not raw:
        return 1.0
    return len(raw) / max(len(zlib.compress(raw, 6)), 1)


def has_repetition(text: str) -> bool:
    """A >10k-char response whose last 10k chars compress more than 10x."""
    if len(text) <= REPETITION_MIN_CHARS:
        return False
    return compression_ratio(text[-REPETITION_MIN_CHARS:]) > REPETITION_COMPRESSION_RATIO


__all__ = ["compression_ratio", "has_repetition"]
