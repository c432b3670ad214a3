"""Request text <-> token ids for the HTTP front.

Without a tokenizer the router keeps the reference's mock scheme (one id per character,
padded to a multiple of 8; `server.tokenize_mock`), which the smoke tests and clients of the
reference rely on. With `LAKE_TOKENIZER=<directory>` (a Hugging Face tokenizer saved next to a
checkpoint: tokenizer.json / tokenizer_config.json) messages are encoded with the model's chat
template when it has one (else the user/system contents joined by newlines) and outputs are
decoded to text. Loading never touches the network.
"""
from __future__ import annotations

import os

from .server import detokenize_mock, tokenize_mock


def _prompt_text(messages) -> str:
    return "\n".join(m.get("content", "") for m in messages or []
                     if isinstance(m, dict) and m.get("role") in ("user", "system"))


class Tokenizer:
    def __init__(self, path: str | None = None):
        self.tok = None
        if path:
            from transformers import AutoTokenizer

            self.tok = AutoTokenizer.from_pretrained(path, local_files_only=True)

    @classmethod
    def from_env(cls) -> "Tokenizer":
        return cls(os.environ.get("LAKE_TOKENIZER") or None)

    @property
    def is_mock(self) -> bool:
        return self.tok is None

    def encode_request(self, data: dict) -> list[int]:
        """Prompt ids of a chat request: explicit `prompt_token_ids`, else the messages."""
        if isinstance(data.get("prompt_token_ids"), list):
            return [int(t) for t in data["prompt_token_ids"]]
        messages = data.get("messages", []) or []
        if self.tok is None:
            return tokenize_mock(_prompt_text(messages))
        msgs = [m for m in messages if isinstance(m, dict) and "content" in m]
        if getattr(self.tok, "chat_template", None):
            return list(self.tok.apply_chat_template(msgs, add_generation_prompt=True, tokenize=True))
        return list(self.tok.encode(_prompt_text(messages)))

    def decode(self, ids) -> str:
        if self.tok is None:
            return detokenize_mock(ids)
        return self.tok.decode(list(ids), skip_special_tokens=True)
