"""Offline engine: request admission, the step loop and ``generate``.

Reference: nanovllm/engine/llm_engine.py:38-532.  Same public surface
(``LLM(model, **Config fields)``, ``add_request``, ``step``, ``generate``,
``cancel_request``, ``metrics``, ``set_scheduler_overlap``, ``exit``) and the
same step semantics:

* serial step: schedule -> run -> postprocess;
* overlap step (``scheduler_overlap=True``): one batch in flight; the next
  batch is scheduled speculatively while the GPU runs the current one, stale
  rows are pruned with the batch's frozen row metadata before launch, and
  turning overlap off drains the pipeline instead of dropping a parked batch;
* admission checks: max_model_len, KV capacity (``OverflowError``), vocab
  range of raw token ids (``ValueError``);
* per-step JSONL trace (``metrics_path``) and engine counters;
* exit watchdog: a wedged teardown kills the worker ranks and exits after
  ``B200MOE_EXIT_TIMEOUT_S`` (or ``NANOVLLM_EXIT_TIMEOUT_S``; 0 disables).
"""
from __future__ import annotations

import atexit
import json
import os
import sys
import threading
from collections import Counter
from time import perf_counter

from tqdm.auto import tqdm

from b200moe.config import Config, config_field_names
from b200moe.engine.executor import Executor
from b200moe.engine.scheduler import ScheduledBatch, Scheduler
from b200moe.engine.sequence import Sequence
from b200moe.sampling_params import SamplingParams
from b200moe.utils.tokenizer import load_tokenizer


def _exit_timeout() -> float:
    return float(os.environ.get("B200MOE_EXIT_TIMEOUT_S", os.environ.get("NANOVLLM_EXIT_TIMEOUT_S", "60")))


class LLMEngine:

    def __init__(self, model: str, **kwargs):
        names = config_field_names()
        config = Config(model, **{k: v for k, v in kwargs.items() if k in names})
        self.config = config
        Sequence.block_size = config.kvcache_block_size
        self.tokenizer = load_tokenizer(model, config.hf_config.vocab_size, config.hf_config.eos_token_id)
        eos = getattr(self.tokenizer, "eos_token_id", None)
        config.eos = eos if eos is not None else (config.hf_config.eos_token_id or -1)
        self.executor = Executor(config)
        self.model_runner = self.executor.runner
        self.scheduler = Scheduler(config)
        if config.kv_offload_enabled:
            for r, bm in enumerate(self.scheduler.block_managers):
                bm.set_offload_executor(self.executor.rank_caller(r) if config.dp_size > 1 else
                                        _AllRanks(self.executor))
        self.last_token_events: list = []
        self.schedule_mode_counts: Counter = Counter()
        self.step_count = 0
        self.prefill_tokens_total = 0
        self.decode_tokens_total = 0
        self.schedule_time_total = 0.0
        self.forward_time_total = 0.0
        self.metrics_path = config.metrics_path
        self.last_step_metrics = None
        self._overlap = bool(config.scheduler_overlap)
        self._pending: ScheduledBatch | None = None
        self._sched_next: ScheduledBatch | None = None
        self._pending_launch_time = 0.0
        self.overlap_defers = 0
        self.overlap_pruned_rows = 0
        # launch-ahead decode (B200MOE_DECODE_FEED=0 disables it)
        self._decode_feed = os.environ.get("B200MOE_DECODE_FEED", "1") != "0"
        self.decode_feed_steps = 0
        self._grammar = None
        self._grammar_cache: dict = {}
        self._exited = False
        atexit.register(self.exit)
        self.kv_outlier_dims = None
        if config.kv_cache_dtype == "int8" and config.kv_int8_mode == "channel":
            self._calibrate_int8_kv()

    def _calibrate_int8_kv(self):
        """int8 channel mode: run a few prompts through every rank with statistics on,
        freeze the per-channel scales and outlier dims, then forget the calibration
        traffic (prefix cache, counters).  The reference does the same at start-up
        with eight mixed-language prompts (nanovllm/engine/llm_engine.py:88-131);
        here the prompts are fixed pseudo-random token ids, as the model may have no
        real tokenizer."""
        import random
        rng = random.Random(1234)
        vocab = self.config.hf_config.vocab_size
        lens = [96, 160, 64, 224, 128, 192, 80, 144]
        cap = max(8, self.config.max_model_len - 32)
        prompts = [[rng.randrange(vocab) for _ in range(min(n, cap))] for n in lens]
        try:
            self.executor.call("kv_calibrate_begin")
            self.generate(prompts, SamplingParams(temperature=0.0, max_tokens=16, ignore_eos=True), use_tqdm=False)
            self.scheduler.clear_prefix_cache()
            self.kv_outlier_dims = self.executor.call("kv_calibrate_freeze")
        except Exception:
            self.exit()
            raise
        self.step_count = 0
        self.schedule_mode_counts.clear()
        self.prefill_tokens_total = self.decode_tokens_total = 0
        self.schedule_time_total = self.forward_time_total = 0.0
        self.last_token_events = []
        self.last_step_metrics = None

    # ------------------------------------------------------------ teardown
    def _force_exit(self):
        print("[engine] exit watchdog fired: teardown still blocked; killing ranks", file=sys.stderr, flush=True)
        for p in getattr(self.executor, "procs", []):
            try:
                p.kill()
            except Exception:
                pass
        # 0 by default (the work is done; only teardown wedged); test runs set a non-zero
        # code so that a wedged teardown cannot end a test process as a success
        os._exit(int(os.environ.get("B200MOE_EXIT_WATCHDOG_RC", "0")))

    def exit(self):
        if self._exited or not hasattr(self, "executor"):
            return
        self._exited = True
        timeout = _exit_timeout()
        watchdog = None
        if timeout > 0:
            watchdog = threading.Timer(timeout, self._force_exit)
            watchdog.daemon = True
            watchdog.start()
        try:
            self.executor.exit()
        finally:
            if watchdog is not None:
                watchdog.cancel()

    # ------------------------------------------------------------ requests
    @property
    def kv_token_capacity(self) -> int:
        return self.config.num_kvcache_blocks * self.config.kvcache_block_size

    def add_request(self, prompt: str | list[int], sampling_params: SamplingParams) -> int:
        if isinstance(prompt, str):
            prompt = self.tokenizer.encode(prompt)
        if not prompt:
            raise ValueError("empty prompt")
        total = len(prompt) + sampling_params.max_tokens
        if total > self.config.max_model_len:
            raise ValueError(f"prompt({len(prompt)}) + max_tokens({sampling_params.max_tokens}) "
                             f"exceeds max_model_len({self.config.max_model_len})")
        if total > self.kv_token_capacity:
            raise OverflowError(f"request needs {total} tokens but KV capacity is {self.kv_token_capacity} tokens")
        vocab = self.config.hf_config.vocab_size
        lo, hi = min(prompt), max(prompt)
        if lo < 0 or hi >= vocab:
            raise ValueError(f"prompt token id {hi if hi >= vocab else lo} outside vocab range [0, {vocab})")
        seq = Sequence(prompt, sampling_params)
        if seq.params.guided_json is not None or seq.params.guided_regex is not None:
            self._attach_grammar(seq)
        self.scheduler.add(seq)
        return seq.seq_id

    def _attach_grammar(self, seq: Sequence):
        """Compile (cached) an xgrammar matcher for a guided request."""
        try:
            import xgrammar as xg
        except ImportError as exc:
            raise ValueError("guided generation requires xgrammar") from exc
        if self._grammar is None:
            info = xg.TokenizerInfo.from_huggingface(self.tokenizer, vocab_size=self.config.hf_config.vocab_size)
            self._grammar = (xg, info, xg.GrammarCompiler(info))
        xg, info, compiler = self._grammar
        if seq.params.guided_json is not None:
            schema = seq.params.guided_json if isinstance(seq.params.guided_json, str) else json.dumps(seq.params.guided_json, sort_keys=True)
            key, build = ("json", schema), (lambda: compiler.compile_json_schema(schema))
        else:
            key, build = ("regex", seq.params.guided_regex), (lambda: compiler.compile_regex(seq.params.guided_regex))
        compiled = self._grammar_cache.get(key)
        if compiled is None:
            compiled = self._grammar_cache[key] = build()
        seq.grammar = xg.GrammarMatcher(compiled)

    def cancel_request(self, seq_id: int) -> bool:
        return self.scheduler.cancel(seq_id)

    # -------------------------------------- prefill / decode disaggregation
    def prefilled_sequences(self) -> list[Sequence]:
        """Running sequences whose prompt is computed and that hold their first
        generated token: ready to hand off to a decode engine."""
        return [s for s in self.scheduler.running if not s.is_finished and not s.in_prefill
                and s.output_len >= 1]

    def detach(self, seq: Sequence):
        """Stop scheduling a handed-off sequence but keep its KV blocks (they
        are read by an in-flight transfer); ``release`` frees them."""
        self.scheduler.running.remove(seq)

    def release(self, seq: Sequence):
        from b200moe.engine.sequence import SequenceStatus
        if seq.block_table:
            self.scheduler._bm(seq).deallocate(seq)
        seq.finish("handoff")

    def admit_prefilled(self, token_ids: list[int], num_prompt_tokens: int,
                        sampling_params: SamplingParams) -> Sequence | None:
        """Decode side of a handoff: reserve KV blocks for a sequence whose KV
        (all tokens but the last) comes from a prefill engine.  Returns None
        while the pool lacks room (back-pressure); after the KV import, call
        ``activate``."""
        seq = Sequence(list(token_ids), sampling_params)
        seq.prompt_len = num_prompt_tokens
        bm = self.scheduler.block_manager
        if bm.num_free_blocks < seq.num_blocks:
            return None
        for _ in range(seq.num_blocks):
            seq.block_table.append(bm._allocate_block())
        seq.dp_rank = 0
        seq.in_prefill = False
        return seq

    def activate(self, seq: Sequence):
        """Start decoding a handed-off sequence whose KV has been imported.
        Its full blocks join the prefix cache (their KV is exactly a local
        prefill's), with the chained hashes a local prefill would give."""
        from b200moe.engine.sequence import SequenceStatus
        bm = self.scheduler.block_manager
        seq.cached_len = 0
        bm.hash_blocks(seq, seq.num_tokens - 1)
        seq.cached_len = seq.num_tokens - 1
        seq.status = SequenceStatus.RUNNING
        seq.timing.stamp(perf_counter())
        self.scheduler.running.append(seq)

    def set_scheduler_overlap(self, enabled: bool):
        """Runtime switch; disabling drains the pipeline (parked batch launches)."""
        self._overlap = bool(enabled)

    # ----------------------------------------------------------- profiling
    def set_profiling(self, enabled: bool):
        """Start or stop the device-timed ranges on every rank."""
        self.executor.call("set_profiling", bool(enabled))

    def start_profiling(self):
        self.set_profiling(True)

    def stop_profiling(self):
        self.set_profiling(False)

    def profile_snapshot(self, reset: bool = True) -> dict:
        """Every rank's per-range p50 / p95 (reference: nanovllm/engine/model_runner.py:377-383
        gathers the ranks' snapshots).  ``max_over_ranks`` keeps, per range,
        the slowest rank's figures: a step waits for its slowest rank."""
        per_rank = self.executor.call_all("profile_snapshot", reset)
        worst: dict[str, dict] = {}
        for snap in per_rank:
            for name, st in snap["segments"].items():
                w = worst.setdefault(name, {"count": 0, "total_ms": 0.0, "p50_ms": 0.0, "p95_ms": 0.0})
                for key in w:
                    w[key] = max(w[key], st[key])
        return {"ranks": per_rank, "max_over_ranks": worst}

    # --------------------------------------------------------------- steps
    def _grammar_masks(self, batch: ScheduledBatch):
        """Allowed-token bitmask per guided row (batch row -> int32 words)."""
        if not any(s.grammar is not None for s in batch.sequences):
            return None
        import torch
        words = (self.config.hf_config.vocab_size + 31) // 32
        masks = {}
        for i, s in enumerate(batch.sequences):
            if s.grammar is not None:
                buf = torch.zeros(1, words, dtype=torch.int32)
                s.grammar.fill_next_token_bitmask(buf, 0)
                masks[i] = buf[0].numpy().copy()
        return masks

    def _launch(self, batch: ScheduledBatch, feed_from: ScheduledBatch | None = None):
        self._pending_launch_time = perf_counter()
        self.executor.launch(batch, self._grammar_masks(batch), feed_from)

    def _feedable(self, nxt: ScheduledBatch, cur: ScheduledBatch) -> bool:
        """Launch-ahead decode: the next decode batch can be enqueued before the
        current one's tokens are read back when every row continues a row of
        the current decode batch (its input token is read on the device) and
        nothing on the host depends on the token values in between: greedy
        sampling, no penalties, log-probs or grammar constraints."""
        if not self._decode_feed or cur.mode != "decode" or nxt.mode != "decode" or any(nxt.prefill_flags):
            return False
        live = {id(s) for s in cur.sequences}
        for s in nxt.sequences:
            if (id(s) not in live or s.params.temperature >= 1e-3 or s.penalty is not None or s.params.logprobs
                    or s.grammar is not None):
                return False
        return True

    def step(self):
        self.last_token_events = []
        if self._overlap or self._pending is not None or self._sched_next is not None:
            return self._step_overlap()
        batch = self.scheduler.schedule()
        if not batch.sequences:
            self.last_step_metrics = {"mode": "empty", "schedule_s": batch.schedule_s, "forward_s": 0.0}
            return [], 0
        self._launch(batch)
        token_ids, logprobs = self.executor.collect()
        return self._finish_step(batch, token_ids, logprobs)

    def _step_overlap(self):
        if (self._pending is not None and self._sched_next is not None
                and self._feedable(self._sched_next, self._pending)):
            # launch-ahead: enqueue step N+1 (decode rows read N's tokens on the device),
            # then read back and apply step N while N+1 runs.  Rows of sequences that
            # finish at N run once more in N+1; their tokens are dropped by postprocess.
            nxt, self._sched_next = self._sched_next, None
            self._launch(nxt, feed_from=self._pending)
            token_ids, logprobs = self.executor.collect()
            outputs, num_tokens = self._finish_step(self._pending, token_ids, logprobs)
            self._pending = nxt
            spec = self.scheduler.schedule(speculative=True, inflight=nxt.sequences)
            if spec.mode == "defer":
                self.overlap_defers += 1
            self._sched_next = None if (spec.mode == "defer" or not spec.sequences) else spec
            self.decode_feed_steps += 1
            return outputs, num_tokens
        outputs, num_tokens = [], 0
        collected = False
        if self._pending is not None:
            token_ids, logprobs = self.executor.collect()
            outputs, num_tokens = self._finish_step(self._pending, token_ids, logprobs)
            self._pending = None
            collected = True
        batch = self._sched_next
        self._sched_next = None
        if batch is not None:
            batch = self._prune_batch(batch)
        elif self._overlap:
            batch = self.scheduler.schedule()
        if batch is None or batch.mode == "defer" or not batch.sequences:
            if not collected:
                self.last_step_metrics = {"mode": "empty", "schedule_s": batch.schedule_s if batch else 0.0,
                                          "forward_s": 0.0}
            return outputs, num_tokens
        self._launch(batch)
        self._pending = batch
        if not collected:
            self.last_step_metrics = {"mode": batch.mode, "schedule_s": batch.schedule_s, "forward_s": 0.0}
        if self._overlap:
            nxt = self.scheduler.schedule(speculative=True, inflight=batch.sequences)
            if nxt.mode == "defer":
                self.overlap_defers += 1
            self._sched_next = None if (nxt.mode == "defer" or not nxt.sequences) else nxt
        return outputs, num_tokens

    def _prune_batch(self, batch: ScheduledBatch) -> ScheduledBatch | None:
        """Drop rows made stale while the batch was parked: finished
        sequences, prefill rows whose last chunk completed in the batch before
        (live ``is_prefill`` cleared), and clamp continuing chunks to the
        tokens actually left.  Uses the frozen row metadata only."""
        kept, flags = [], []
        for seq, q, was_prefill in zip(batch.sequences, batch.query_lens, batch.prefill_flags):
            if seq.is_finished:
                self.overlap_pruned_rows += 1
                continue
            if was_prefill:
                if not seq.in_prefill:
                    self.overlap_pruned_rows += 1
                    seq.chunk_len = 0
                    continue
                q = min(q, seq.num_tokens - seq.cached_len)
            if q <= 0:
                self.overlap_pruned_rows += 1
                seq.chunk_len = 0
                seq.in_prefill = False
                continue
            seq.chunk_len = q
            seq.in_prefill = was_prefill
            kept.append(seq)
            flags.append(was_prefill)
        if not kept:
            return None
        has_dec, has_pre = (not all(flags)), any(flags)
        mode = "mixed" if (has_dec and has_pre) else ("decode" if has_dec else "prefill")
        return ScheduledBatch(kept, [s.chunk_len for s in kept],
                              [s.cached_len + s.chunk_len for s in kept],
                              sum(s.chunk_len for s in kept), mode, batch.schedule_s, flags)

    def _finish_step(self, batch: ScheduledBatch, token_ids, logprobs):
        seqs, mode = batch.sequences, batch.mode
        flags, qlens = batch.prefill_flags, batch.query_lens
        self.schedule_mode_counts[mode] += 1
        prefill_tokens = sum(q for q, f in zip(qlens, flags) if f)
        decode_tokens = sum(q for q, f in zip(qlens, flags) if not f)
        num_tokens = batch.num_scheduled_tokens if mode != "decode" else -len(seqs)
        forward_s = perf_counter() - self._pending_launch_time
        done_before = {id(s) for s in seqs if s.is_finished}  # finished by the previous step (launch-ahead rows)
        self.last_token_events = self.scheduler.postprocess(seqs, token_ids, mode, logprobs, qlens, flags)
        self.step_count += 1
        self.prefill_tokens_total += prefill_tokens
        self.decode_tokens_total += decode_tokens
        self.schedule_time_total += batch.schedule_s
        self.forward_time_total += forward_s
        self.last_step_metrics = {"mode": mode, "schedule_s": batch.schedule_s, "forward_s": forward_s}
        if self.metrics_path:
            rec = {"kind": "step", "step": self.step_count, "mode": mode, "effective_batch": len(seqs),
                   "prefill_tokens": prefill_tokens, "decode_tokens": decode_tokens,
                   "scheduled_tokens": batch.num_scheduled_tokens, "query_lens": qlens,
                   "context_lens": batch.context_lens, "schedule_s": batch.schedule_s, "forward_s": forward_s}
            with open(self.metrics_path, "a", encoding="utf-8") as f:
                f.write(json.dumps(rec, separators=(",", ":")) + "\n")
        outputs = [(s.seq_id, s.output_ids(), s.metrics()) for s in seqs
                   if s.is_finished and id(s) not in done_before]
        return outputs, num_tokens

    # -------------------------------------------------------------- public
    def metrics(self) -> dict:
        m = {
            "engine_steps_total": self.step_count,
            "engine_prefill_tokens_total": self.prefill_tokens_total,
            "engine_decode_tokens_total": self.decode_tokens_total,
            "engine_schedule_seconds_total": self.schedule_time_total,
            "engine_forward_seconds_total": self.forward_time_total,
        }
        for mode, n in self.schedule_mode_counts.items():
            m[f"engine_{mode}_steps_total"] = n
        m["engine_overlap_defers_total"] = self.overlap_defers
        m["engine_overlap_pruned_rows_total"] = self.overlap_pruned_rows
        m["engine_decode_feed_steps_total"] = self.decode_feed_steps
        m.update(self.scheduler.metrics())
        return m

    def is_finished(self) -> bool:
        return self.scheduler.is_finished() and self._pending is None and self._sched_next is None

    def generate(self, prompts: list[str] | list[list[int]],
                 sampling_params: SamplingParams | list[SamplingParams] | None = None,
                 use_tqdm: bool = True) -> list[dict]:
        """Run every prompt to completion; returns ``{"text", "token_ids",
        "metrics"}`` per prompt, in prompt order."""
        sampling_params = sampling_params or SamplingParams()
        if not isinstance(sampling_params, list):
            sampling_params = [sampling_params] * len(prompts)
        ids = [self.add_request(p, sp) for p, sp in zip(prompts, sampling_params)]
        order = {sid: i for i, sid in enumerate(ids)}
        outputs: dict[int, tuple] = {}
        pbar = tqdm(total=len(prompts), desc="Generating", dynamic_ncols=True, disable=not use_tqdm)
        while not self.is_finished():
            t = perf_counter()
            out, num_tokens = self.step()
            dt = max(perf_counter() - t, 1e-9)
            if use_tqdm:
                key = "Prefill" if num_tokens > 0 else "Decode"
                pbar.set_postfix({key: f"{int(abs(num_tokens) / dt)}tok/s"})
            for sid, toks, met in out:
                if sid in order:
                    outputs[sid] = (toks, met)
                    pbar.update(1)
        pbar.close()
        res = []
        for sid in ids:
            toks, met = outputs[sid]
            res.append({"text": self.tokenizer.decode(toks), "token_ids": toks, "metrics": met})
        return res


class _AllRanks:
    """Offload executor for a single shared block table: every rank moves its own KV share."""

    def __init__(self, executor: Executor):
        self.executor = executor

    def call(self, method, *args):
        return self.executor.call(method, *args)
