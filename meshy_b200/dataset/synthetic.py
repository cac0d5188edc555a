"""Synthetic prompts for benchmarks and tests (no data download).

``SyntheticPrompts`` yields random token-id prompts with uniform lengths and a
seeded parity rule reward, matching the BASELINE configs ("prompts = random
token ids, binary rule reward with p = 0.5").
"""

from __future__ import annotations

import random

from ..utils.sample import Sample


class SyntheticPrompts:
    def __init__(self, batch_size: int, n_prompts: int = 100_000, vocab_size: int = 151936, min_len: int = 64,
                 max_len: int = 512, seed: int = 0, target_token: int | None = None):
        self.batch_size = batch_size
        self.n_prompts = n_prompts
        self.vocab_size = vocab_size
        self.min_len, self.max_len = min_len, max_len
        self.seed = seed
        self.index = 0
        self.target_token = target_token

    def seek(self, index: int) -> None:
        self.index = int(index)

    def _prompt(self, i: int) -> list[int]:
        r = random.Random(self.seed * 1_000_003 + i)
        return [r.randrange(self.vocab_size) for _ in range(r.randint(self.min_len, self.max_len))]

    def next_batch(self, builder) -> list[Sample]:
        if self.index + self.batch_size > self.n_prompts:
            return []
        out = []
        for i in range(self.index, self.index + self.batch_size):
            s = builder.from_tokens(self._prompt(i), ground_truth=self.target_token)
            s.prompt_id = i
            out.append(s)
        self.index += self.batch_size
        return out

    @staticmethod
    def reward(sample) -> float:
        """1 if the response holds the target token (when set) else parity of the response id sum."""
        resp = [t for t, m in zip(sample.tokens, sample.masks) if m]
        if sample.ground_truth is not None:
            return 1.0 if int(sample.ground_truth) in resp else 0.0
        return 1.0 if sum(resp) % 2 == 0 else 0.0


__all__ = ["SyntheticPrompts"]
