"""Local-file math datasets with the reference's prompt templates and graders.

* :class:`MATH`: DAPO-Math-17k rows (``prompt`` = chat messages, ``reward_model.ground_truth``), scored by
  DAPO's strict boxed check (``+1`` / ``-1``), as ``meshy/dataset/math.py`` does. Plain rows
  (``problem`` / ``question`` text with ``answer`` / ``solution``) are read too.
* :class:`GSM8K`: ``question`` / ``answer`` rows, the ``####`` prompt and the numeric ``####`` match
  (``meshy/dataset/gsm8k.py``).
* :class:`S9Math`: S9 records, ``prompt`` = a non-empty message list and ``label`` = the answer, graded by
  :func:`~meshy_b200.dataset.math_reward.math_reward` (``meshy/dataset/s9_math.py``); prompts longer than
  ``prompt_max_tokens`` are an error.

This framework never downloads: the path comes from the constructor or the dataset's environment variable
(``MATH_DATASET_PATH``, ``GSM8K_DATASET_PATH``, ``S9_DATASET_PATH``).
"""

from __future__ import annotations

import os
from typing import Any

from .base import Dataset
from .math_reward import dapo_compute_score, gsm8k_answer, gsm8k_reward, math_reward

PROMPT_SUFFIX = "\n\nPlease reason step by step, and put your final answer within \\boxed{}."
GSM8K_SUFFIX = " Let's think step by step and output the final answer after \"####\"."


def _last_response(sample) -> str:
    return sample.messages[-1]["content"] if sample.messages else ""


class MATH(Dataset):
    def __init__(self, batch_size: int, seed: int | None = None, path: str | None = None, limit: int | None = None):
        path = path or os.environ.get("MATH_DATASET_PATH", "")
        super().__init__(self.read_jsonl(path) if path else [], batch_size, seed, limit)

    def apply_chat_template(self, row: dict, builder):
        prompt = row.get("prompt")
        if isinstance(prompt, list) and prompt:  # DAPO-17k: chat messages + reward_model.ground_truth
            question = prompt[0]["content"]
            truth = (row.get("reward_model") or {}).get("ground_truth", row.get("answer"))
        else:
            question = prompt or row.get("problem") or row.get("question")
            truth = row.get("answer") or row.get("solution")
        s = builder.build_sample([{"role": "user", "content": question + PROMPT_SUFFIX}])
        s.ground_truth = truth
        return s

    @staticmethod
    def reward(sample) -> float:
        return float(dapo_compute_score(_last_response(sample), str(sample.ground_truth),
                                        strict_box_verify=True)["score"])


class GSM8K(Dataset):
    def __init__(self, batch_size: int, seed: int | None = None, path: str | None = None, limit: int | None = None):
        path = path or os.environ.get("GSM8K_DATASET_PATH", "")
        super().__init__(self.read_jsonl(path) if path else [], batch_size, seed, limit)

    def apply_chat_template(self, row: dict, builder):
        s = builder.build_sample([{"role": "system", "content": "You are a helpful assistant."},
                                  {"role": "user", "content": row["question"] + GSM8K_SUFFIX}])
        s.ground_truth = gsm8k_answer(row["answer"])
        return s

    @staticmethod
    def reward(sample) -> float:
        return gsm8k_reward(_last_response(sample), sample.ground_truth)


class S9Math(Dataset):
    def __init__(self, batch_size: int, seed: int | None = None, path: str | None = None, limit: int | None = None,
                 prompt_max_tokens: int = 2048):
        if batch_size <= 0:
            raise ValueError("batch_size must be positive")
        if prompt_max_tokens <= 0:
            raise ValueError("prompt_max_tokens must be positive")
        path = path or os.environ.get("S9_DATASET_PATH", "")
        rows = self._read(path) if path else []
        super().__init__(rows, batch_size, seed, limit)
        self.prompt_max_tokens = int(prompt_max_tokens)

    @staticmethod
    def _read(path: str) -> list[dict[str, Any]]:
        import json

        if not os.path.isfile(path):
            raise FileNotFoundError(f"S9 dataset not found: {path}")
        rows = []
        with open(path, encoding="utf-8") as f:
            for n, line in enumerate(f, 1):
                if not line.strip():
                    continue
                try:
                    row = json.loads(line)
                except ValueError as e:
                    raise ValueError(f"{path}:{n}: not JSON") from e
                if not isinstance(row, dict) or "prompt" not in row or "label" not in row:
                    raise ValueError(f"{path}:{n}: an S9 record is an object with 'prompt' and 'label'")
                rows.append(row)
        if not rows:
            raise ValueError(f"S9 dataset is empty: {path}")
        return rows

    def apply_chat_template(self, row: dict, builder):
        msgs = row["prompt"]
        if not isinstance(msgs, list) or not msgs:
            raise ValueError("an S9 prompt is a non-empty list of messages")
        clean = []
        for m in msgs:
            if not (isinstance(m, dict) and isinstance(m.get("role"), str) and isinstance(m.get("content"), str)):
                raise ValueError("S9 messages need string 'role' and 'content'")
            clean.append({"role": m["role"], "content": m["content"]})
        s = builder.build_sample(clean)
        if len(s.tokens) > self.prompt_max_tokens:
            raise ValueError(f"S9 prompt has {len(s.tokens)} tokens, more than {self.prompt_max_tokens}")
        s.ground_truth = row["label"]
        return s

    @staticmethod
    def reward(sample) -> float:
        return math_reward(_last_response(sample), sample.ground_truth)


__all__ = ["GSM8K", "MATH", "S9Math"]
