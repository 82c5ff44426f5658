"""Incremental detokenisation for streaming (reference: nanovllm/incremental_detokenizer.py:46-84).

Keeps a window of recent token ids; each ``push`` decodes the window with
and without the new token and emits only the new suffix, holding text back
while it ends in an incomplete UTF-8 sequence (the replacement character).
"""
from __future__ import annotations


class IncrementalDetokenizer:

    def __init__(self, tokenizer, skip_special_tokens: bool = True, window: int = 6):
        self.tokenizer = tokenizer
        self.skip = skip_special_tokens
        self.window = window
        self.ids: list[int] = []
        self.prefix_offset = 0   # start of the decode window
        self.read_offset = 0     # tokens already emitted

    def _decode(self, ids) -> str:
        return self.tokenizer.decode(ids, skip_special_tokens=self.skip)

    def push(self, token_id: int) -> str:
        self.ids.append(int(token_id))
        prefix = self._decode(self.ids[self.prefix_offset:self.read_offset])
        full = self._decode(self.ids[self.prefix_offset:])
        if full.endswith("�") or len(full) <= len(prefix):
            return ""
        delta = full[len(prefix):]
        self.read_offset = len(self.ids)
        if self.read_offset - self.prefix_offset > self.window:
            self.prefix_offset = self.read_offset - self.window // 2
        return delta

    def flush(self) -> str:
        prefix = self._decode(self.ids[self.prefix_offset:self.read_offset])
        full = self._decode(self.ids[self.prefix_offset:])
        self.read_offset = len(self.ids)
        return full[len(prefix):] if len(full) > len(prefix) else ""
