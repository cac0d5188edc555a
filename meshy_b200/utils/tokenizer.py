"""Tokenizers for the sample builder.

* :class:`ByteChatTokenizer` — dependency-free byte-level tokenizer with a
  ChatML-style template (ids 0-3 special, bytes at 4..259).  Used for
  synthetic runs and tests; no download needed.
* :func:`load_tokenizer` — a local HF tokenizer directory (``local_files_only``)
  or the byte tokenizer for ``"synthetic"`` / unreachable paths.
"""

from __future__ import annotations

import os

PAD, BOS, EOS, IM_START, IM_END = 0, 1, 2, 3, 2
_OFF = 4


class ByteChatTokenizer:
    eos_token_id = EOS
    pad_token_id = PAD
    vocab_size = 256 + _OFF

    def encode(self, text: str) -> list[int]:
        return [b + _OFF for b in text.encode("utf-8")]

    def decode(self, ids, skip_special_tokens: bool = True) -> str:
        return bytes(int(i) - _OFF for i in ids if _OFF <= int(i) < _OFF + 256).decode("utf-8", errors="replace")

    def apply_chat_template(self, messages, tokenize: bool = True, add_generation_prompt: bool = False):
        ids: list[int] = []
        for m in messages:
            ids += [IM_START] + self.encode(f"{m['role']}\n{m['content']}") + [IM_END] + self.encode("\n")
        if add_generation_prompt:
            ids += [IM_START] + self.encode("assistant\n")
        return ids


def load_tokenizer(model_path: str | None):
    if not model_path or model_path == "synthetic" or not os.path.isdir(str(model_path)):
        return ByteChatTokenizer()
    try:
        from transformers import AutoTokenizer

        return AutoTokenizer.from_pretrained(model_path, local_files_only=True)
    except Exception:
        return ByteChatTokenizer()


__all__ = ["ByteChatTokenizer", "load_tokenizer"]
