"""Rollout samples and the chat-template-aware builder.

``SampleBuilder`` renders messages to token spans by prefix diffing (each
message's ids are the difference between successive renders without the
generation prompt), so masks mark exactly the assistant tokens (reference
``meshy/utils/sample.py:8-122``).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Iterable

from .tokenizer import load_tokenizer


@dataclass
class Sample:
    messages: list = field(default_factory=list)
    tokens: list = field(default_factory=list)
    logprobs: list = field(default_factory=list)
    masks: list = field(default_factory=list)
    ground_truth: Any = None
    reward: float | None = None
    advantage: float | None = None
    raw_reward: float | None = None
    finish_reason: str | None = None
    truncated: bool = False
    repetition: bool = False
    mixed_version: bool = False
    positive_lm_weight: float = 0.0
    prompt_id: int = -1


class SampleBuilder:
    def __init__(self, model_path: str | None = None, tokenizer=None):
        self.tokenizer = tokenizer or load_tokenizer(model_path)

    def _render(self, messages, *, add_generation_prompt: bool) -> list[int]:
        if not messages:
            return []
        out = self.tokenizer.apply_chat_template(messages, tokenize=True, add_generation_prompt=add_generation_prompt)
        return list(out["input_ids"] if hasattr(out, "keys") else out)

    def _spans(self, messages):
        spans, prev = [], []
        for i, m in enumerate(messages):
            full = self._render(messages[: i + 1], add_generation_prompt=False)
            spans.append((m["role"], full[len(prev):]))
            prev = full
        spans.append((None, self._render(messages, add_generation_prompt=True)[len(prev):]))
        return spans

    def build_sample(self, messages: Iterable[dict], logprob: float = 0.0) -> Sample:
        messages = [{"role": m["role"], "content": m["content"]} for m in messages]
        s = Sample(messages=messages)
        for role, ids in self._spans(messages):
            s.tokens.extend(ids)
            s.logprobs.extend([logprob] * len(ids))
            s.masks.extend([1 if role == "assistant" else 0] * len(ids))
        return s

    def from_tokens(self, prompt_ids: Iterable[int], ground_truth: Any = None) -> Sample:
        ids = list(prompt_ids)
        return Sample(messages=[{"role": "user", "content": ""}], tokens=ids, logprobs=[0.0] * len(ids),
                      masks=[0] * len(ids), ground_truth=ground_truth)

    def append_text(self, sample: Sample, role: str, content: str, logprob: float = 0.0, *,
                    add_generation_prompt: bool = True) -> Sample:
        old = self._render(list(sample.messages), add_generation_prompt=False)
        new_msgs = [*sample.messages, {"role": role, "content": content}]
        new = self._render(new_msgs, add_generation_prompt=add_generation_prompt)
        if new[: len(old)] != old:
            raise ValueError("chat template changed the existing message prefix")
        sample.messages.append({"role": role, "content": content})
        ids = new[len(old):]
        sample.tokens.extend(ids)
        sample.logprobs.extend([logprob] * len(ids))
        sample.masks.extend([1 if role == "assistant" else 0] * len(ids))
        return sample

    def append_tokens(self, sample: Sample, role: str, tokens: Iterable[int], logprobs: Iterable[float]) -> Sample:
        tokens = list(tokens)
        sample.messages.append({"role": role, "content": self.tokenizer.decode(tokens, skip_special_tokens=True)})
        sample.tokens.extend(tokens)
        sample.logprobs.extend(list(logprobs))
        sample.masks.extend([1 if role == "assistant" else 0] * len(tokens))
        return sample


__all__ = ["Sample", "SampleBuilder"]
