"""Continuous-batching scheduler.

Policies and invariants follow the reference Scheduler
(nanovllm/engine/scheduler.py:35-483):

* ``fcfs``: prefill-first; decode only when no prefill is admissible; only the
  first sequence of a step may be chunked by the token budget.
* ``stall_free``: decode-first, then bounded prefill chunks
  (``prefill_chunk_size``) fill the remaining budget; a candidate whose KV
  cannot be admitted is skipped (no head-of-line blocking) and re-queued in
  order; a chunked sequence is picked at most once per step.
* ``stall_free_lpm``: as stall_free, but inside a priority tier the waiting
  sequence with the longest cached prefix is admitted first (probing does not
  touch the LRU).
* priority tiers (lower value first) with a starvation guard
  (``scheduler_starvation_steps``), priority-aware recompute preemption, cancel,
  and the overlap pipeline's speculative pass (never preempts; defers when the
  cumulative launch-time block shortfall does not fit).

B200 extension, data-parallel attention: with ``dp_size`` > 1 every rank owns
a private KV pool, so there is one :class:`BlockManager` per rank; a sequence
is bound to a rank on admission (best prefix hit, then most free token budget,
then most free blocks) and the token / sequence budgets apply per rank.
Preemption victims come from the requester's rank.  With ``dp_size == 1`` the
decisions are exactly the single-pool ones.
"""
from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field
from time import perf_counter

from b200moe.engine.block_manager import BlockManager
from b200moe.engine.sequence import Sequence, SequenceStatus


@dataclass(slots=True)
class ScheduledBatch:
    sequences: list[Sequence]
    query_lens: list[int]
    context_lens: list[int]
    num_scheduled_tokens: int
    mode: str
    schedule_s: float = 0.0
    # row phase frozen at schedule time (the overlap pipeline rewrites the
    # live fields for the next batch while this one is in flight)
    prefill_flags: list[bool] = field(default_factory=list)

    def __iter__(self):
        yield self.sequences
        yield self.mode


class Scheduler:

    def __init__(self, config, dp_size: int | None = None):
        self.max_num_seqs = config.max_num_seqs
        self.max_num_batched_tokens = config.max_num_batched_tokens
        self.eos = config.eos
        self.block_size = config.kvcache_block_size
        self.policy = config.scheduler_policy
        self.prefill_chunk_size = config.prefill_chunk_size
        self.starvation_steps = config.scheduler_starvation_steps
        self.dp_size = dp_size if dp_size is not None else getattr(config, "dp_size", 1)
        self.block_managers = [BlockManager(config.num_kvcache_blocks, config.kvcache_block_size)
                               for _ in range(self.dp_size)]
        self.waiting: deque[Sequence] = deque()
        self.running: deque[Sequence] = deque()
        self.preemptions = 0
        self.kv_admission_skips_total = 0

    @property
    def block_manager(self) -> BlockManager:
        return self.block_managers[0]

    def _bm(self, seq: Sequence) -> BlockManager:
        return self.block_managers[max(seq.dp_rank, 0)]

    def is_finished(self) -> bool:
        return not self.waiting and not self.running

    def add(self, seq: Sequence):
        self.waiting.append(seq)

    def cancel(self, seq_id: int) -> bool:
        for queue in (self.waiting, self.running):
            for seq in queue:
                if seq.seq_id != seq_id:
                    continue
                queue.remove(seq)
                if seq.block_table:
                    self._bm(seq).deallocate(seq)
                seq.finish("cancelled")
                return True
        return False

    # ------------------------------------------------------------ schedule
    def schedule(self, speculative: bool = False, inflight: list | None = None) -> ScheduledBatch:
        """``speculative=True`` is the overlap pipeline's pass one step ahead of
        the GPU: sequences in ``inflight`` grow by one token before this batch
        launches, and the pass defers instead of preempting."""
        t0 = perf_counter()
        if self.policy == "fcfs":
            seqs, mode = self._schedule_fcfs(speculative, inflight)
        else:
            seqs, mode = self._schedule_stall_free(speculative, inflight)
        if mode in ("defer", "empty"):
            return ScheduledBatch([], [], [], 0, mode, perf_counter() - t0)
        return ScheduledBatch(
            sequences=seqs,
            query_lens=[s.chunk_len for s in seqs],
            context_lens=[s.cached_len + s.chunk_len for s in seqs],
            num_scheduled_tokens=sum(s.chunk_len for s in seqs),
            mode=mode,
            schedule_s=perf_counter() - t0,
            prefill_flags=[s.in_prefill for s in seqs],
        )

    def _speculative_precheck(self, inflight) -> tuple[bool, dict]:
        """Read-only pass over the decode rows the speculative schedule will
        take (same order and budgets): defer when their cumulative launch-time
        block shortfall does not fit a rank's free pool."""
        inflight_ids = {id(s) for s in (inflight or [])}
        launch_len: dict[int, int] = {}
        budgets = [self.max_num_batched_tokens] * self.dp_size
        counts = [0] * self.dp_size
        checked: list[list[Sequence]] = [[] for _ in range(self.dp_size)]
        for seq in self.running:
            r = max(seq.dp_rank, 0)
            if budgets[r] == 0 or counts[r] >= self.max_num_seqs:
                if self.dp_size == 1:
                    break
                continue
            checked[r].append(seq)
            launch_len[id(seq)] = len(seq) + (1 if id(seq) in inflight_ids else 0)
            budgets[r] -= 1
            counts[r] += 1
        for r, seqs in enumerate(checked):
            bm = self.block_managers[r]
            if seqs and bm.total_launch_shortfall(seqs, [launch_len[id(s)] for s in seqs]) > bm.num_free_blocks:
                return True, launch_len
        return False, launch_len

    def _decode_pass(self, speculative: bool, launch_len: dict, budgets: list[int] | None) -> list[Sequence]:
        """Schedule running sequences for one decode token each, preempting on
        KV shortage (never in a speculative pass).  ``budgets`` (per-rank
        token budget) is decremented when given.  Leaves ``self.running`` as
        scheduled rows + rows not reached, in order."""
        scheduled: list[Sequence] = []
        skipped: list[Sequence] = []
        counts = [0] * self.dp_size
        while self.running:
            seq = self.running[0]
            r = max(seq.dp_rank, 0)
            full = counts[r] >= self.max_num_seqs or (budgets is not None and budgets[r] == 0)
            if full:
                if self.dp_size == 1:
                    break
                skipped.append(self.running.popleft())
                continue
            self.running.popleft()
            bm = self._bm(seq)
            if speculative:
                bm.may_append_at(seq, launch_len.get(id(seq), len(seq)))
            else:
                preempted_self = False
                while not bm.can_append(seq):
                    victim = self._preempt_victim(requester=seq)
                    if victim is None:
                        self.preempt(seq)
                        preempted_self = True
                        break
                    self.preempt(victim)
                if preempted_self:
                    continue
                bm.may_append(seq)
            seq.chunk_len = 1
            seq.in_prefill = False
            scheduled.append(seq)
            counts[r] += 1
            if budgets is not None:
                budgets[r] -= 1
        self.running.extendleft(reversed(skipped))
        return scheduled

    def _probe_rank(self, seq: Sequence, budgets: list[int], counts: list[int]):
        """(rank, cached_blocks) for a new sequence, or None if no rank fits."""
        best = None
        for r, bm in enumerate(self.block_managers):
            if budgets[r] <= 0 or counts[r] >= self.max_num_seqs:
                continue
            n = bm.can_allocate(seq, touch=False)
            if n < 0:
                continue
            key = (n, budgets[r], bm.num_free_blocks, -r)
            if best is None or key > best[0]:
                best = (key, r, n)
        return None if best is None else (best[1], best[2])

    def _allocate_on(self, seq: Sequence, r: int):
        seq.dp_rank = r
        bm = self.block_managers[r]
        bm.allocate(seq, bm.can_allocate(seq))  # touch-on-hit for the real admission

    def _schedule_fcfs(self, speculative: bool, inflight):
        launch_len: dict = {}
        if speculative:
            defer, launch_len = self._speculative_precheck(inflight)
            if defer:
                return [], "defer"
        scheduled: list[Sequence] = []
        budgets = [self.max_num_batched_tokens] * self.dp_size
        counts = [0] * self.dp_size
        while self.waiting and sum(counts) < self.max_num_seqs * self.dp_size:
            seq = self.waiting[0]
            seq.timing.mark_scheduled(perf_counter())
            if not seq.block_table:
                if max(budgets) == 0:
                    break
                probe = self._probe_rank(seq, budgets, counts)
                if probe is None:
                    break
                r, cached = probe
                num_tokens = seq.num_tokens - cached * self.block_size
                if budgets[r] < num_tokens and counts[r] > 0:  # only a step's first seq is chunked
                    break
                self._allocate_on(seq, r)
            else:
                r = max(seq.dp_rank, 0)
                if budgets[r] == 0 or counts[r] >= self.max_num_seqs:
                    break
                num_tokens = seq.num_tokens - seq.cached_len
                if budgets[r] < num_tokens and counts[r] > 0:
                    break
            seq.chunk_len = min(num_tokens, budgets[r])
            budgets[r] -= seq.chunk_len
            counts[r] += 1
            if seq.cached_len + seq.chunk_len == seq.num_tokens:
                seq.status = SequenceStatus.RUNNING
                self.waiting.popleft()
                self.running.append(seq)
            scheduled.append(seq)
        if scheduled:
            return scheduled, "prefill"
        scheduled = self._decode_pass(speculative, launch_len, None)
        if not scheduled:
            return [], "empty"
        self.running.extendleft(reversed(scheduled))
        return scheduled, "decode"

    def _waiting_candidate(self, touch: bool = False) -> Sequence:
        """Highest priority first; FIFO within a tier (lpm: longest cached
        prefix).  Sequences waiting ``starvation_steps`` passes outrank all."""
        starved = [s for s in self.waiting if s.wait_steps >= self.starvation_steps]
        if starved:
            cand = max(starved, key=lambda s: (s.wait_steps, -s.params.priority))
        else:
            cand = min(self.waiting, key=lambda s: s.params.priority)
            if self.policy == "stall_free_lpm":
                tier = [s for s in self.waiting if s.params.priority == cand.params.priority]
                if len(tier) > 1:
                    def cached_blocks(s):
                        if s.block_table:
                            return s.cached_len // self.block_size
                        return max(bm.can_allocate(s, touch=touch) for bm in self.block_managers)
                    cand = max(tier, key=cached_blocks)
        self.waiting.remove(cand)
        return cand

    def _preempt_victim(self, requester: Sequence | None) -> Sequence | None:
        """Newest lowest-priority running sequence (on the requester's rank);
        None when every candidate outranks the requester."""
        rank = None if requester is None or self.dp_size == 1 else max(requester.dp_rank, 0)
        idx = None
        for i, s in enumerate(self.running):
            if rank is not None and max(s.dp_rank, 0) != rank:
                continue
            if idx is None or s.params.priority >= self.running[idx].params.priority:
                idx = i
        if idx is None:
            return None
        victim = self.running[idx]
        if requester is not None and victim.params.priority < requester.params.priority:
            return None
        del self.running[idx]
        return victim

    def _schedule_stall_free(self, speculative: bool, inflight):
        launch_len: dict = {}
        if speculative:
            defer, launch_len = self._speculative_precheck(inflight)
            if defer:
                return [], "defer"
        budgets = [self.max_num_batched_tokens] * self.dp_size
        decode = self._decode_pass(speculative, launch_len, budgets)
        counts = [0] * self.dp_size
        for s in decode:
            counts[max(s.dp_rank, 0)] += 1
        for seq in self.waiting:
            seq.wait_steps += 1
        prefill: list[Sequence] = []
        skipped: list[Sequence] = []
        requeued: list[Sequence] = []
        for _ in range(len(self.waiting)):
            if not self.waiting:
                break
            if max(budgets) == 0 or all(c >= self.max_num_seqs for c in counts):
                break
            seq = self._waiting_candidate()
            seq.timing.mark_scheduled(perf_counter())
            if not seq.block_table:
                probe = self._probe_rank(seq, budgets, counts)
                if probe is None:
                    skipped.append(seq)
                    self.kv_admission_skips_total += 1
                    continue
                self._allocate_on(seq, probe[0])
            r = max(seq.dp_rank, 0)
            if budgets[r] == 0 or counts[r] >= self.max_num_seqs:
                skipped.append(seq)
                continue
            remaining = seq.num_tokens - seq.cached_len
            seq.chunk_len = min(remaining, budgets[r], self.prefill_chunk_size)
            seq.wait_steps = 0
            budgets[r] -= seq.chunk_len
            counts[r] += 1
            prefill.append(seq)
            if seq.cached_len + seq.chunk_len == seq.num_tokens:
                seq.status = SequenceStatus.RUNNING
                self.running.append(seq)
            else:
                requeued.append(seq)
        for seq in reversed(skipped):
            self.waiting.appendleft(seq)
        self.waiting.extend(requeued)
        self.running.extendleft(reversed(decode))
        scheduled = decode + prefill
        if not scheduled:
            return [], "empty"
        if decode and prefill:
            return scheduled, "mixed"
        return scheduled, ("decode" if decode else "prefill")

    def preempt(self, seq: Sequence):
        self.preemptions += 1
        seq.status = SequenceStatus.WAITING
        seq.in_prefill = True
        self._bm(seq).deallocate(seq)
        if self.dp_size > 1:
            seq.dp_rank = -1
        self.waiting.appendleft(seq)

    def clear_prefix_cache(self):
        """Drop every cached (unreferenced) prefix block on every rank."""
        for bm in self.block_managers:
            bm.clear_prefix_cache()

    def metrics(self) -> dict:
        m = dict(self.block_managers[0].metrics())
        for bm in self.block_managers[1:]:
            for k, v in bm.metrics().items():
                if k != "kv_lru_enabled":
                    m[k] = m[k] + v
        if self.dp_size > 1:
            cap = m["kv_blocks_capacity"]
            m["kv_cache_utilization"] = m["kv_blocks_used"] / cap if cap else 0.0
        m.update({
            "scheduler_waiting_requests": len(self.waiting),
            "scheduler_running_requests": len(self.running),
            "scheduler_preemptions_total": self.preemptions,
            "scheduler_kv_admission_skips_total": self.kv_admission_skips_total,
        })
        return m

    def _remove_from_queues(self, seq: Sequence):
        if seq in self.waiting:
            self.waiting.remove(seq)
        if seq in self.running:
            self.running.remove(seq)

    def postprocess(self, seqs: list[Sequence], token_ids: list[int], mode: str,
                    logprobs: list | None = None, query_lens: list[int] | None = None,
                    prefill_flags: list[bool] | None = None):
        """Apply one batch's sampled tokens using the batch's FROZEN row
        metadata (``query_lens`` / ``prefill_flags``).  Returns token events
        ``(seq_id, token, finished, metrics|None, logprobs|None)``."""
        if query_lens is None:
            query_lens = [s.chunk_len for s in seqs]
        if prefill_flags is None:
            prefill_flags = [s.in_prefill for s in seqs]
        events = []
        for row, (seq, tok) in enumerate(zip(seqs, token_ids)):
            if seq.is_finished:
                continue
            q = query_lens[row]
            was_prefill = prefill_flags[row]
            seq.in_prefill = was_prefill
            bm = self._bm(seq)
            bm.hash_blocks(seq, q)
            seq.cached_len += q
            seq.chunk_len = 0
            if was_prefill and seq.cached_len < seq.num_tokens:
                continue
            seq.append(tok)
            if was_prefill:
                seq.in_prefill = False
            now = perf_counter()
            seq.timing.stamp(now)
            hit_eos = not seq.params.ignore_eos and tok == self.eos
            hit_stop = seq.params.stop_token_ids is not None and tok in seq.params.stop_token_ids
            hit_grammar = False
            if seq.grammar is not None:
                seq.grammar.accept_token(tok)
                hit_grammar = seq.grammar.is_terminated()
            hit_len = seq.output_len == seq.params.max_tokens
            if hit_eos or hit_stop or hit_grammar or hit_len:
                seq.finish("stop" if (hit_eos or hit_stop or hit_grammar) else "length", now)
                bm.deallocate(seq)
                self._remove_from_queues(seq)
            elif was_prefill and seq in self.waiting:
                self.waiting.remove(seq)
                self.running.append(seq)
                seq.status = SequenceStatus.RUNNING
            events.append((seq.seq_id, tok, seq.is_finished,
                           seq.metrics() if seq.is_finished else None,
                           logprobs[row] if logprobs is not None else None))
        return events
