"""Prompt datasets: ``next_batch(builder) -> [Sample]`` with a seekable ``index``.

Datasets read local files only (this framework never downloads).  The
rollout checkpoints ``index`` and restores it with :meth:`seek`
(reference ``meshy/dataset/base.py:8-25``).
"""

from __future__ import annotations

import json
import random
from typing import Any


class Dataset:
    def __init__(self, rows: list[dict], batch_size: int, seed: int | None = None, limit: int | None = None):
        self.rows = list(rows)
        if seed is not None:
            random.Random(seed).shuffle(self.rows)
        if limit is not None:  # a bounded run (smoke / fixture recipes): the first ``limit`` prompts only
            self.rows = self.rows[:int(limit)]
        self.batch_size = int(batch_size)
        self.index = 0

    @property
    def n_prompts(self) -> int:
        return len(self.rows)

    def seek(self, index: int) -> None:
        self.index = int(index)

    def next_batch(self, builder) -> list:
        if self.index + self.batch_size > len(self.rows):
            return []
        batch = self.rows[self.index:self.index + self.batch_size]
        self.index += self.batch_size
        return [self.apply_chat_template(r, builder) for r in batch]

    def apply_chat_template(self, row: dict, builder):
        raise NotImplementedError

    @staticmethod
    def read_jsonl(path: str) -> list[dict]:
        with open(path, encoding="utf-8") as f:
            return [json.loads(l) for l in f if l.strip()]


__all__ = ["Dataset"]
