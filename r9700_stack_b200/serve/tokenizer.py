"""Tokenizers for the server.

Synthetic checkpoints have no vocabulary, so the default is a byte-level tokenizer (UTF-8 bytes
shifted past a few special ids). A local Hugging Face tokenizer directory can be given instead
(``HFTokenizer``); nothing is downloaded.
"""
from __future__ import annotations


class ByteTokenizer:
    PAD, BOS, EOS = 0, 1, 2
    OFFSET = 3

    def __init__(self, vocab_size: int = 512):
        assert vocab_size >= 256 + self.OFFSET
        self.vocab_size = vocab_size
        self.eos_token_id = self.EOS

    def encode(self, text: str) -> list[int]:
        return [b + self.OFFSET for b in text.encode("utf-8")]

    def decode(self, ids: list[int]) -> str:
        bs = bytes(i - self.OFFSET for i in ids if self.OFFSET <= i < 256 + self.OFFSET)
        return bs.decode("utf-8", errors="replace")

    def apply_chat_template(self, messages: list[dict]) -> str:
        parts = [f"<|{m.get('role', 'user')}|>\n{m.get('content', '')}\n" for m in messages]
        return "".join(parts) + "<|assistant|>\n"


class HFTokenizer:
    def __init__(self, path: str):
        from transformers import AutoTokenizer

        self.tok = AutoTokenizer.from_pretrained(path, local_files_only=True)
        self.eos_token_id = self.tok.eos_token_id if self.tok.eos_token_id is not None else -1
        self.vocab_size = len(self.tok)

    def encode(self, text: str) -> list[int]:
        return self.tok.encode(text, add_special_tokens=False)

    def decode(self, ids: list[int]) -> str:
        return self.tok.decode(ids, skip_special_tokens=True)

    def apply_chat_template(self, messages: list[dict]) -> str:
        return self.tok.apply_chat_template(messages, tokenize=False, add_generation_prompt=True)
