"""Chat tokenisation for recipes.

Reference: the tokeniser processors of ``axrl/processor`` (chat template, appended-message tokens,
run in the processor pool).  :class:`ChatTokenizer` wraps a Hugging Face tokenizer loaded from a
LOCAL path (``local_files_only``) and renders messages with its chat template.  :class:`ByteTokenizer`
is a dependency-free stand-in (UTF-8 bytes + a ChatML-like template) for tests and synthetic runs.

``append_message_ids`` returns the ids that extend an already-rendered conversation by one message
(tool observations, user turns) so multi-turn rollouts grow the token stream without re-rendering.
"""

from __future__ import annotations

from typing import Any


class ByteTokenizer:
    """ids: 0 pad, 1 <|im_start|>, 2 <|im_end|>, 3 eos; byte b -> 16 + b."""

    pad_id, im_start, im_end, eos_id = 0, 1, 2, 3
    vocab_size = 16 + 256

    def encode(self, text: str) -> list[int]:
        return [16 + b for b in text.encode("utf-8")]

    def decode(self, ids: list[int]) -> str:
        return bytes(i - 16 for i in ids if 16 <= i < 272).decode("utf-8", errors="replace")

    def _msg(self, role: str, content: str) -> list[int]:
        return [self.im_start] + self.encode(f"{role}\n{content}") + [self.im_end] + self.encode("\n")

    def apply_chat_template(self, messages: list[dict], add_generation_prompt: bool = True, tools: Any = None) -> list[int]:
        ids: list[int] = []
        for m in messages:
            ids += self._msg(m["role"], m.get("content") or "")
        if add_generation_prompt:
            ids += [self.im_start] + self.encode("assistant\n")
        return ids


class ChatTokenizer:
    def __init__(self, path_or_tokenizer: Any) -> None:
        if isinstance(path_or_tokenizer, str):
            from transformers import AutoTokenizer

            self.tok = AutoTokenizer.from_pretrained(path_or_tokenizer, local_files_only=True, trust_remote_code=False)
        else:
            self.tok = path_or_tokenizer
        self.eos_id = getattr(self.tok, "eos_token_id", None) or getattr(self.tok, "eos_id", 0)

    def render(self, messages: list[dict], tools: list[dict] | None = None, add_generation_prompt: bool = True) -> list[int]:
        if isinstance(self.tok, ByteTokenizer):
            return self.tok.apply_chat_template(messages, add_generation_prompt, tools)
        out = self.tok.apply_chat_template(messages, tools=tools, add_generation_prompt=add_generation_prompt, tokenize=True)
        return list(out["input_ids"] if isinstance(out, dict) else out)

    def decode(self, ids: list[int]) -> str:
        return self.tok.decode(list(ids), skip_special_tokens=True) if not isinstance(self.tok, ByteTokenizer) else self.tok.decode(ids)

    def append_message_ids(self, role: str, content: str, add_generation_prompt: bool = True) -> list[int]:
        """Tokens that extend a rendered conversation (ending after an assistant turn) by one message."""
        if isinstance(self.tok, ByteTokenizer):
            ids = self.tok._msg(role, content)
            return ids + ([self.tok.im_start] + self.tok.encode("assistant\n") if add_generation_prompt else [])
        base = [{"role": "user", "content": "x"}, {"role": "assistant", "content": "y"}]
        a = self.render(base, add_generation_prompt=False)
        b = self.render(base + [{"role": role, "content": content}], add_generation_prompt=add_generation_prompt)
        assert b[:len(a)] == a, "chat template does not extend by appending"
        return b[len(a):]
