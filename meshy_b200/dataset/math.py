"""Local-file math datasets: GSM8K (``####`` answers), MATH / DAPO-17k (boxed), S9 JSONL."""

from __future__ import annotations

import os

from .base import Dataset
from .math_reward import boxed_reward, gsm8k_reward

PROMPT_SUFFIX = "\nPlease reason step by step, and put your final answer within \\boxed{}."


class MATH(Dataset):
    """Rows ``{"prompt"|"problem": str, "answer"|"solution": str}`` from a local JSONL."""

    def __init__(self, batch_size: int, seed: int | None = None, path: str | None = None, limit: int | None = None):
        path = path or os.environ.get("MATH_DATASET_PATH", "")
        super().__init__(self.read_jsonl(path) if path else [], batch_size, seed, limit)

    def apply_chat_template(self, row, builder):
        q = row.get("prompt") or row.get("problem") or row.get("question")
        s = builder.build_sample([{"role": "user", "content": q + PROMPT_SUFFIX}])
        s.ground_truth = row.get("answer") or row.get("solution")
        return s

    @staticmethod
    def reward(sample) -> float:
        return boxed_reward(sample.messages[-1]["content"] if sample.messages else "", sample.ground_truth)


class GSM8K(Dataset):
    def __init__(self, batch_size: int, seed: int | None = None, path: str | None = None, limit: int | None = None):
        path = path or os.environ.get("GSM8K_DATASET_PATH", "")
        super().__init__(self.read_jsonl(path) if path else [], batch_size, seed, limit)

    def apply_chat_template(self, row, builder):
        s = builder.build_sample([{"role": "user", "content": row["question"] + PROMPT_SUFFIX}])
        s.ground_truth = row["answer"]
        return s

    @staticmethod
    def reward(sample) -> float:
        return gsm8k_reward(sample.messages[-1]["content"] if sample.messages else "", sample.ground_truth)


class S9Math(MATH):
    def __init__(self, batch_size: int, seed: int | None = None, path: str | None = None, limit: int | None = None):
        super().__init__(batch_size, seed, path or os.environ.get("S9_DATASET_PATH", ""), limit)


__all__ = ["GSM8K", "MATH", "S9Math"]
