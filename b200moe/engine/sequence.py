"""The driver's record of one request.

Worker ranks never see this object: the driver packs what a step needs into a
flat plan (``engine/step_plan.py``).  So the record is organised around its
three readers on the driver:

* the scheduler and block manager: token ids, the KV block table and the
  prefill cursor (``cached_len`` tokens already in KV, ``chunk_len`` tokens in
  the step being launched);
* the plan packer: the request's :class:`SamplingParams` (held as given, not
  copied field by field) and, only when a penalty is set, a
  :class:`PenaltyCounts`;
* metrics: a :class:`RequestTiming`, whose ``report`` produces the per-request
  dict the reference's benchmark readers expect (keys of
  nanovllm/engine/sequence.py ``metrics``).
"""
from __future__ import annotations

import enum
import itertools
from dataclasses import dataclass, field
from time import perf_counter

from b200moe.sampling_params import SamplingParams


class SequenceStatus(enum.IntEnum):
    WAITING = 0
    RUNNING = 1
    FINISHED = 2


@dataclass(slots=True)
class RequestTiming:
    """Host timestamps of one request (``perf_counter`` seconds)."""
    arrival: float = field(default_factory=perf_counter)
    scheduled: float | None = None   # first time a step included it
    finished: float | None = None
    stamps: list[float] = field(default_factory=list)  # one per output token

    def stamp(self, t: float):
        self.stamps.append(t)

    def mark_scheduled(self, t: float):
        if self.scheduled is None:
            self.scheduled = t

    def report(self, prompt_tokens: int, output_tokens: int, finish_reason: str | None) -> dict:
        first = self.stamps[0] if self.stamps else None
        end = self.finished if self.finished is not None else (self.stamps[-1] if self.stamps else None)
        since = lambda t: None if t is None else t - self.arrival
        ttft, e2e = since(first), since(end)
        per_token = None
        if ttft is not None and e2e is not None and output_tokens > 1:
            per_token = (e2e - ttft) / (output_tokens - 1)
        intervals = [b - a for a, b in itertools.pairwise(self.stamps)]
        return {"prompt_tokens": prompt_tokens, "output_tokens": output_tokens, "queue_s": since(self.scheduled),
                "ttft_s": ttft, "e2e_s": e2e, "tpot_s": per_token, "mean_tpot_s": per_token,
                "itls_s": intervals, "token_intervals_s": intervals, "finish_reason": finish_reason}


class PenaltyCounts:
    """Token occurrence counts for presence / frequency / repetition penalties.

    ``generated`` counts output tokens (presence and frequency penalties).  The
    repetition penalty also looks at the prompt; that table is built on first
    use from the prompt as it stands then, so a prefilled hand-over that moves
    the prompt boundary before any step is still counted right."""
    __slots__ = ("generated", "_seen")

    def __init__(self):
        self.generated: dict[int, int] = {}
        self._seen: dict[int, int] | None = None

    def add(self, token: int):
        self.generated[token] = self.generated.get(token, 0) + 1
        if self._seen is not None:
            self._seen[token] = self._seen.get(token, 0) + 1

    def seen(self, prompt) -> dict[int, int]:
        if self._seen is None:
            table: dict[int, int] = {}
            for t in prompt:
                table[t] = table.get(t, 0) + 1
            for t, c in self.generated.items():
                table[t] = table.get(t, 0) + c
            self._seen = table
        return self._seen


def _wants_penalty(sp: SamplingParams) -> bool:
    return sp.presence_penalty != 0.0 or sp.frequency_penalty != 0.0 or sp.repetition_penalty != 1.0


class Sequence:
    """One request: tokens, KV blocks, prefill cursor, sampling and timing."""

    block_size = 256           # KV block size; the engine sets it from its config
    _ids = itertools.count()

    __slots__ = ("seq_id", "status", "tokens", "prompt_len", "cached_len", "chunk_len", "in_prefill",
                 "block_table", "params", "penalty", "grammar", "timing", "wait_steps", "finish_reason",
                 "dp_rank")

    def __init__(self, token_ids: list[int], sampling_params: SamplingParams | None = None):
        self.seq_id = next(Sequence._ids)
        self.status = SequenceStatus.WAITING
        self.tokens = list(token_ids)
        self.prompt_len = len(self.tokens)
        self.cached_len = 0          # tokens whose KV is in the pool
        self.chunk_len = 0           # tokens the current step computes
        self.in_prefill = True
        self.block_table: list[int] = []
        self.params = sampling_params or SamplingParams()
        self.penalty = PenaltyCounts() if _wants_penalty(self.params) else None
        self.grammar = None          # xgrammar matcher of a guided request
        self.timing = RequestTiming()
        self.wait_steps = 0          # scheduler passes spent waiting (starvation guard)
        self.finish_reason: str | None = None
        self.dp_rank = -1            # data-parallel rank owning the KV (-1 = unassigned)

    # ------------------------------------------------------------------ tokens
    def __len__(self) -> int:
        return len(self.tokens)

    @property
    def num_tokens(self) -> int:
        return len(self.tokens)

    @property
    def last(self) -> int:
        return self.tokens[-1]

    @property
    def output_len(self) -> int:
        return len(self.tokens) - self.prompt_len

    def output_ids(self) -> list[int]:
        return self.tokens[self.prompt_len:]

    def prompt_ids(self) -> list[int]:
        return self.tokens[:self.prompt_len]

    def append(self, token: int):
        self.tokens.append(token)
        if self.penalty is not None:
            self.penalty.add(token)

    # ------------------------------------------------------------------ blocks
    @property
    def num_blocks(self) -> int:
        return -(-len(self.tokens) // self.block_size)

    def block_tokens(self, i: int) -> list[int]:
        """Token ids held by logical block ``i`` (the last may be partial)."""
        if i < 0 or i >= self.num_blocks:
            raise IndexError(f"block {i} of a {self.num_blocks}-block sequence")
        lo = i * self.block_size
        return self.tokens[lo:lo + self.block_size]

    # ------------------------------------------------------------------ status
    @property
    def is_finished(self) -> bool:
        return self.status is SequenceStatus.FINISHED

    def finish(self, reason: str, t: float | None = None):
        self.status = SequenceStatus.FINISHED
        self.finish_reason = reason
        self.timing.finished = perf_counter() if t is None else t

    def metrics(self) -> dict:
        return self.timing.report(self.prompt_len, self.output_len, self.finish_reason)
