"""Rollout samples, and turning chat messages into token spans with loss masks.

A :class:`Sample` is one trajectory: its messages, the token ids the policy
saw, a per-token behaviour log-prob, and a per-token mask that is 1 exactly on
assistant tokens (the tokens the loss trains). Its field names are the
column names the rollout publishes, as in the reference
(``meshy/utils/sample.py``).

Chat templates are not compositional token by token, so the token ids of
message ``i`` are found by rendering the conversation up to and including
``i`` and keeping what that render adds to the render up to ``i - 1``. The
trailing generation prompt (``<|im_start|>assistant`` and the like) is the
part that the final render *with* ``add_generation_prompt`` adds, and it
belongs to the prompt (mask 0).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Iterable, Iterator

from .tokenizer import load_tokenizer

ASSISTANT = "assistant"


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

    def extend(self, ids: list[int], *, trained: bool, logprobs: Iterable[float] | float = 0.0) -> None:
        """Append ``ids`` with their behaviour log-probs (one per id, or one value for all) and mask."""
        lps = [float(logprobs)] * len(ids) if isinstance(logprobs, (int, float)) else [float(x) for x in logprobs]
        if len(lps) != len(ids):
            raise ValueError(f"{len(ids)} tokens but {len(lps)} log-probs")
        self.tokens += ids
        self.logprobs += lps
        self.masks += [int(trained)] * len(ids)


def _ids(rendered) -> list[int]:
    """Token ids of a ``apply_chat_template(tokenize=True)`` result (a list, or a BatchEncoding)."""
    if isinstance(rendered, (list, tuple)):
        return list(rendered)
    ids = rendered["input_ids"] if "input_ids" in rendered else rendered
    return list(ids)


class SampleBuilder:
    def __init__(self, model_path: str | None = None, tokenizer=None):
        self.tokenizer = tokenizer if tokenizer is not None else load_tokenizer(model_path)

    def render(self, messages: list[dict], generation_prompt: bool) -> list[int]:
        if not messages:
            return []
        return _ids(self.tokenizer.apply_chat_template(messages, tokenize=True,
                                                       add_generation_prompt=generation_prompt))

    def segments(self, messages: list[dict]) -> Iterator[tuple[str | None, list[int]]]:
        """``(role, ids)`` of every message, then ``(None, generation-prompt ids)``."""
        done: list[int] = []
        for k in range(len(messages)):
            upto = self.render(messages[:k + 1], False)
            yield messages[k]["role"], upto[len(done):]
            done = upto
        yield None, self.render(messages, True)[len(done):]

    def build_sample(self, messages: Iterable[dict], logprob: float = 0.0) -> Sample:
        msgs = [{"role": m["role"], "content": m["content"]} for m in messages]
        sample = Sample(messages=msgs)
        for role, ids in self.segments(msgs):
            sample.extend(ids, trained=role == ASSISTANT, logprobs=logprob)
        return sample

    def from_tokens(self, prompt_ids: Iterable[int], ground_truth: Any = None) -> Sample:
        """A prompt given as token ids (no chat template; one empty user message stands for it)."""
        sample = Sample(messages=[{"role": "user", "content": ""}], ground_truth=ground_truth)
        sample.extend(list(prompt_ids), trained=False)
        return sample

    def append_text(self, sample: Sample, role: str, content: str, logprob: float = 0.0, *,
                    add_generation_prompt: bool = True) -> Sample:
        """Add one message rendered through the template; the existing render must stay a prefix."""
        before = self.render(list(sample.messages), False)
        msg = {"role": role, "content": content}
        after = self.render([*sample.messages, msg], add_generation_prompt)
        if after[:len(before)] != before:
            raise ValueError("the chat template re-rendered earlier messages differently; cannot append")
        sample.messages.append(msg)
        sample.extend(after[len(before):], trained=role == ASSISTANT, logprobs=logprob)
        return sample

    def append_tokens(self, sample: Sample, role: str, tokens: Iterable[int], logprobs: Iterable[float]) -> Sample:
        """Add generated tokens verbatim (the engine's ids and log-probs); the message text is their decode."""
        ids = list(tokens)
        text = self.tokenizer.decode(ids, skip_special_tokens=True)
        sample.messages.append({"role": role, "content": text})
        sample.extend(ids, trained=role == ASSISTANT, logprobs=list(logprobs))
        return sample


__all__ = ["Sample", "SampleBuilder"]
