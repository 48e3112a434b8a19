"""Tokenizers for the rollout server and the chat-completion entry points.

A local Hugging Face checkpoint directory with tokenizer files uses its own
tokenizer and chat template (``transformers.AutoTokenizer``).  Without one
(preset architectures with random weights: benchmarks, tests, this offline
image) :class:`ByteTokenizer` is used: UTF-8 bytes are ids 0..255 and three
control tokens follow (``<|im_start|>``, ``<|im_end|>``, ``<|endoftext|>``),
with a ChatML-style template, so any model whose vocabulary has at least 259
entries can serve chat requests end to end.
"""

from __future__ import annotations

import json
import os
from typing import Any, Protocol


class Tokenizer(Protocol):
    eos_token_ids: list[int]

    def encode(self, text: str) -> list[int]: ...

    def decode(self, ids: list[int]) -> str: ...

    def apply_chat_template(self, messages: list[dict[str, Any]], tools: list | None = None,
                            add_generation_prompt: bool = True) -> list[int]: ...


class ByteTokenizer:
    IM_START, IM_END, EOT = 256, 257, 258

    def __init__(self) -> None:
        self.eos_token_ids = [self.IM_END, self.EOT]

    def encode(self, text: str) -> list[int]:
        return list(text.encode("utf-8"))

    def decode(self, ids: list[int]) -> str:
        return bytes(i for i in ids if 0 <= i < 256).decode("utf-8", errors="replace")

    def token_str(self, i: int) -> str:
        if i == self.IM_START:
            return "<|im_start|>"
        if i == self.IM_END:
            return "<|im_end|>"
        if i == self.EOT:
            return "<|endoftext|>"
        return bytes([i]).decode("latin-1") if 0 <= i < 256 else f"<{i}>"

    def apply_chat_template(self, messages: list[dict[str, Any]], tools: list | None = None,
                            add_generation_prompt: bool = True) -> list[int]:
        ids: list[int] = []
        if tools:
            ids += [self.IM_START] + self.encode("system\n# Tools\n" + json.dumps(tools)) + [self.IM_END]
            ids += self.encode("\n")
        for m in messages:
            content = m.get("content") or ""
            if isinstance(content, list):  # content parts
                content = "".join(p.get("text", "") for p in content if isinstance(p, dict))
            body = f"{m.get('role', 'user')}\n{content}"
            if m.get("tool_calls"):
                body += "\n" + json.dumps(m["tool_calls"], default=str)
            ids += [self.IM_START] + self.encode(body) + [self.IM_END] + self.encode("\n")
        if add_generation_prompt:
            ids += [self.IM_START] + self.encode("assistant\n")
        return ids


class HFTokenizer:
    def __init__(self, path: str) -> None:
        from transformers import AutoTokenizer

        self.tok = AutoTokenizer.from_pretrained(path)
        eos = self.tok.eos_token_id
        self.eos_token_ids = [eos] if isinstance(eos, int) else list(eos or [])

    def encode(self, text: str) -> list[int]:
        return self.tok.encode(text, add_special_tokens=False)

    def decode(self, ids: list[int]) -> str:
        return self.tok.decode(ids, skip_special_tokens=True)

    def token_str(self, i: int) -> str:
        return self.tok.convert_ids_to_tokens(i)

    def apply_chat_template(self, messages: list[dict[str, Any]], tools: list | None = None,
                            add_generation_prompt: bool = True) -> list[int]:
        out = self.tok.apply_chat_template(messages, tools=tools, add_generation_prompt=add_generation_prompt,
                                           tokenize=True)
        return list(out["input_ids"] if isinstance(out, dict) else out)


def get_tokenizer(base_model: str) -> ByteTokenizer | HFTokenizer:
    if os.path.isdir(base_model) and any(
        os.path.exists(os.path.join(base_model, f)) for f in ("tokenizer.json", "tokenizer_config.json")
    ):
        return HFTokenizer(base_model)
    return ByteTokenizer()
