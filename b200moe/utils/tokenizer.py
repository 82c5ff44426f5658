"""Tokenizer loading.

A checkpoint directory with HF tokenizer files gets ``AutoTokenizer``.  Without
them (random-init presets, synthetic benchmarks: there is no network to fetch a
vocabulary) a byte-level stand-in is used: ids 0..255 are bytes, the rest map
to printable placeholders, so text in/out round-trips for ASCII and every id in
the model's vocabulary decodes to something.
"""
from __future__ import annotations

import os


class ByteTokenizer:
    """Minimal HF-compatible tokenizer over bytes (ids < 256)."""

    def __init__(self, vocab_size: int, eos_token_id: int | None):
        self.vocab_size = vocab_size
        self.eos_token_id = eos_token_id if eos_token_id is not None else vocab_size - 1
        self.bos_token_id = None
        self.pad_token_id = self.eos_token_id
        self.all_special_ids = [self.eos_token_id]
        self.chat_template = None

    def __len__(self):
        return self.vocab_size

    def encode(self, text: str, add_special_tokens: bool = False) -> list[int]:
        return [b % self.vocab_size for b in text.encode("utf-8")]

    def __call__(self, text, **kw):
        return {"input_ids": self.encode(text)}

    def decode(self, ids, skip_special_tokens: bool = False) -> str:
        out = bytearray()
        for t in ids:
            t = int(t)
            if skip_special_tokens and t in self.all_special_ids:
                continue
            if t < 256:
                out.append(t)
            else:
                out.extend(f"<{t}>".encode())
        return out.decode("utf-8", errors="replace")

    def convert_ids_to_tokens(self, ids):
        return [self.decode([i]) for i in ids]

    def apply_chat_template(self, messages, tokenize: bool = True, add_generation_prompt: bool = True, **kw):
        text = "".join(f"<|{m.get('role', 'user')}|>\n{m.get('content', '')}\n" for m in messages)
        if add_generation_prompt:
            text += "<|assistant|>\n"
        return self.encode(text) if tokenize else text


def load_tokenizer(model: str, vocab_size: int, eos_token_id: int | None):
    if os.path.isdir(model) and any(os.path.exists(os.path.join(model, f))
                                    for f in ("tokenizer.json", "tokenizer_config.json", "vocab.json")):
        try:
            from transformers import AutoTokenizer
            return AutoTokenizer.from_pretrained(model, use_fast=True)
        except Exception:
            pass
    return ByteTokenizer(vocab_size, eos_token_id)
