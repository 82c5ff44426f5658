"""Per-request state (reference: nanovllm/engine/sequence.py:16-173).

Holds token ids, the KV block table, cached/scheduled token counts, sampling
knobs, penalty counters and request timing.  ``metrics()`` returns the same
keys as the reference so benchmark readers carry over.  Worker ranks never see
a ``Sequence``: the driver ships them a flat step plan instead.
"""
from __future__ import annotations

from collections import Counter
from enum import Enum, auto
from itertools import count
from time import perf_counter

from b200moe.sampling_params import SamplingParams


class SequenceStatus(Enum):
    WAITING = auto()
    RUNNING = auto()
    FINISHED = auto()


class Sequence:
    block_size = 256
    counter = count()

    def __init__(self, token_ids: list[int], sampling_params: SamplingParams | None = None):
        sp = sampling_params or SamplingParams()
        self.seq_id = next(Sequence.counter)
        self.status = SequenceStatus.WAITING
        self.token_ids = list(token_ids)
        self.last_token = self.token_ids[-1]
        self.num_tokens = len(self.token_ids)
        self.num_prompt_tokens = len(self.token_ids)
        self.num_cached_tokens = 0
        self.num_scheduled_tokens = 0
        self.is_prefill = True
        self.block_table: list[int] = []
        self.temperature = sp.temperature
        self.max_tokens = sp.max_tokens
        self.ignore_eos = sp.ignore_eos
        self.priority = sp.priority
        self.top_p = sp.top_p
        self.top_k = sp.top_k
        self.min_p = sp.min_p
        self.presence_penalty = sp.presence_penalty
        self.frequency_penalty = sp.frequency_penalty
        self.repetition_penalty = sp.repetition_penalty
        self.logprobs = sp.logprobs or 0
        self.stop_token_ids = tuple(sp.stop_token_ids or ())
        self.guided_json = sp.guided_json
        self.guided_regex = sp.guided_regex
        self.seed = sp.seed
        self.grammar_matcher = None
        self.gen_counts: dict[int, int] = {}
        self.rep_counts: dict[int, int] | None = None
        self.arrival_time = perf_counter()
        self.first_scheduled_time: float | None = None
        self.first_token_time: float | None = None
        self.finish_time: float | None = None
        self.token_times: list[float] = []
        self.wait_steps = 0
        self.finish_reason: str | None = None
        # data-parallel attention: rank that owns this sequence's KV (-1 = unassigned)
        self.dp_rank = -1

    def __len__(self):
        return self.num_tokens

    def __getitem__(self, key):
        return self.token_ids[key]

    @property
    def is_finished(self) -> bool:
        return self.status == SequenceStatus.FINISHED

    @property
    def num_completion_tokens(self) -> int:
        return self.num_tokens - self.num_prompt_tokens

    @property
    def prompt_token_ids(self) -> list[int]:
        return self.token_ids[:self.num_prompt_tokens]

    @property
    def completion_token_ids(self) -> list[int]:
        return self.token_ids[self.num_prompt_tokens:]

    @property
    def num_blocks(self) -> int:
        return (self.num_tokens + self.block_size - 1) // self.block_size

    @property
    def last_block_num_tokens(self) -> int:
        return self.num_tokens - (self.num_blocks - 1) * self.block_size

    @property
    def has_penalty(self) -> bool:
        return (self.presence_penalty != 0.0 or self.frequency_penalty != 0.0
                or self.repetition_penalty != 1.0)

    def ensure_rep_counts(self) -> dict[int, int]:
        """Prompt+generated counts for repetition_penalty, built lazily so a
        PD handoff that rewrites ``num_prompt_tokens`` stays correct."""
        if self.rep_counts is None:
            self.rep_counts = dict(Counter(self.prompt_token_ids))
            for t, c in self.gen_counts.items():
                self.rep_counts[t] = self.rep_counts.get(t, 0) + c
        return self.rep_counts

    def block(self, i: int) -> list[int]:
        if not 0 <= i < self.num_blocks:
            raise IndexError(i)
        return self.token_ids[i * self.block_size:(i + 1) * self.block_size]

    def append_token(self, token_id: int):
        self.token_ids.append(token_id)
        self.last_token = token_id
        self.num_tokens += 1
        self.gen_counts[token_id] = self.gen_counts.get(token_id, 0) + 1
        if self.rep_counts is not None:
            self.rep_counts[token_id] = self.rep_counts.get(token_id, 0) + 1

    def record_token(self, timestamp: float):
        if self.first_token_time is None:
            self.first_token_time = timestamp
        self.token_times.append(timestamp)

    def metrics(self) -> dict:
        finish = self.finish_time or (self.token_times[-1] if self.token_times else None)
        ttft = None if self.first_token_time is None else self.first_token_time - self.arrival_time
        e2e = None if finish is None else finish - self.arrival_time
        gaps = [b - a for a, b in zip(self.token_times, self.token_times[1:])]
        tpot = None
        if e2e is not None and ttft is not None and self.num_completion_tokens > 1:
            tpot = (e2e - ttft) / (self.num_completion_tokens - 1)
        queue = None if self.first_scheduled_time is None else self.first_scheduled_time - self.arrival_time
        return {
            "prompt_tokens": self.num_prompt_tokens,
            "output_tokens": self.num_completion_tokens,
            "queue_s": queue,
            "ttft_s": ttft,
            "e2e_s": e2e,
            "tpot_s": tpot,
            "mean_tpot_s": tpot,
            "itls_s": gaps,
            "token_intervals_s": gaps,
            "finish_reason": self.finish_reason,
        }
