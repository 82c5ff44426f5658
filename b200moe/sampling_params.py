"""Per-request sampling knobs with the reference's defaults and validation
(nanovllm/sampling_params.py:5-61): temperature 0 is greedy, top_k -1 is off,
penalties follow OpenAI (presence/frequency on generated tokens) and vLLM/HF
(repetition on prompt+generated) semantics, logprobs are capped at 20."""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(slots=True)
class SamplingParams:
    temperature: float = 1.0
    max_tokens: int = 64
    ignore_eos: bool = False
    priority: int = 0
    top_p: float = 1.0
    top_k: int = -1
    min_p: float = 0.0
    presence_penalty: float = 0.0
    frequency_penalty: float = 0.0
    repetition_penalty: float = 1.0
    stop_token_ids: tuple[int, ...] | list[int] | None = None
    logprobs: int | None = None
    skip_special_tokens: bool = True
    guided_json: dict | str | None = None
    guided_regex: str | None = None
    seed: int | None = None

    def __post_init__(self):
        if self.temperature < 0:
            raise ValueError("temperature must be non-negative (0 = greedy)")
        if self.priority < 0:
            raise ValueError("priority must be non-negative (0 = highest)")
        if self.max_tokens < 1:
            raise ValueError("max_tokens must be >= 1")
        if not 0.0 < self.top_p <= 1.0:
            raise ValueError("top_p must be in (0, 1]")
        if self.top_k == 0 or self.top_k < -1:
            raise ValueError("top_k must be -1 (disabled) or a positive integer")
        if not 0.0 <= self.min_p <= 1.0:
            raise ValueError("min_p must be in [0, 1]")
        if not -2.0 <= self.presence_penalty <= 2.0:
            raise ValueError("presence_penalty must be in [-2, 2]")
        if not -2.0 <= self.frequency_penalty <= 2.0:
            raise ValueError("frequency_penalty must be in [-2, 2]")
        if not 0.0 < self.repetition_penalty <= 2.0:
            raise ValueError("repetition_penalty must be in (0, 2]")
        if self.logprobs is not None and not 0 <= int(self.logprobs) <= 20:
            raise ValueError("logprobs must be an integer in [0, 20]")
        if self.guided_json is not None and not isinstance(self.guided_json, (dict, str)):
            raise ValueError("guided_json must be a JSON-schema dict or string")
        if self.guided_json is not None and self.guided_regex is not None:
            raise ValueError("guided_json and guided_regex are mutually exclusive")
        if self.guided_regex is not None and not isinstance(self.guided_regex, str):
            raise ValueError("guided_regex must be a string")
        if self.stop_token_ids is not None:
            ok = isinstance(self.stop_token_ids, (list, tuple)) and all(
                isinstance(t, int) and not isinstance(t, bool) for t in self.stop_token_ids)
            if not ok:
                raise ValueError("stop_token_ids must be a list of integers")
            self.stop_token_ids = tuple(self.stop_token_ids)

    @property
    def is_greedy(self) -> bool:
        return self.temperature < 1e-3
