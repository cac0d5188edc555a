"""Sample building and rollout quality stamps (CPU, built-in byte-level ChatML tokenizer).

The builder's tokens equal a full chat-template render with the generation prompt, and its masks cover the
assistant spans only (the trailing generation prompt belongs to the prompt); the repetition stamp flags
looping responses, never prose or short text."""

import random

import pytest

from meshy_b200.utils.metric import compression_ratio, has_repetition
from meshy_b200.utils.sample import SampleBuilder


@pytest.fixture(scope="module")
def builder():
    return SampleBuilder()


@pytest.mark.parametrize("messages", [
    [{"role": "user", "content": "Hi"}],
    [{"role": "system", "content": "You are terse."}, {"role": "user", "content": "Hi"}],
    [{"role": "user", "content": "What is 2+2?"}, {"role": "assistant", "content": "4"},
     {"role": "user", "content": "And 3+3?"}],
])
def test_tokens_match_full_render(builder, messages):
    s = builder.build_sample(messages)
    full = builder.tokenizer.apply_chat_template(messages, tokenize=True, add_generation_prompt=True)
    full = full["input_ids"] if isinstance(full, dict) else list(full)
    assert s.tokens == full
    assert len(s.masks) == len(s.tokens) == len(s.logprobs)


def test_masks_cover_assistant_spans_only(builder):
    msgs = [{"role": "system", "content": "S"}, {"role": "user", "content": "U"},
            {"role": "assistant", "content": "A"}, {"role": "user", "content": "V"}]
    s = builder.build_sample(msgs)
    text = builder.tokenizer.decode([t for t, m in zip(s.tokens, s.masks) if m == 1])
    assert "A" in text and "assistant" in text
    assert not any(c in text for c in "SUV")
    assert s.masks[-1] == 0


def test_repetition_stamp():
    rng = random.Random(0)
    words = ["theorem", "let", "x", "be", "prime", "then", "sum", "over", "k", "modulo", "hence", "we"]
    prose = " ".join(rng.choice(words) + str(rng.randint(0, 999)) for _ in range(6000))
    assert len(prose) > 10_000 and not has_repetition(prose)
    loop = "Therefore the answer is 42. " * 2000
    assert has_repetition(loop) and compression_ratio(loop) > 10
    assert not has_repetition("abc " * 100)  # short responses are never flagged
