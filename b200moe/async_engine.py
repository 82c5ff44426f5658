"""Background engine for online serving (reference: nanovllm/async_engine.py:14-210).

One engine thread owns the :class:`LLMEngine`; the asyncio side talks to it
through a command queue (``add`` / ``cancel`` / ``close``) and per-request
event queues of :class:`TokenEvent`.  Admission control: a full request queue
or a request that can never fit the KV pool raises ``OverflowError`` (HTTP
429); an over-long or out-of-vocab request raises ``ValueError`` (HTTP 400).
If a step raises, every in-flight request receives an error event and the
engine keeps serving.
"""
from __future__ import annotations

import asyncio
import time
from dataclasses import dataclass
from queue import Empty, Queue
from threading import Lock, Thread

from b200moe.engine.llm_engine import LLMEngine
from b200moe.prometheus_metrics import PrometheusMetrics
from b200moe.sampling_params import SamplingParams


@dataclass(slots=True)
class TokenEvent:
    token_id: int | None = None
    finished: bool = False
    cancelled: bool = False
    metrics: dict | None = None
    error: str | None = None
    logprobs: dict | None = None


@dataclass(slots=True)
class RequestHandle:
    seq_id: int
    events: Queue


class AsyncLLMEngine:

    def __init__(self, model: str | None = None, engine: LLMEngine | None = None, **kwargs):
        self.max_queue_size = kwargs.pop("max_queue_size", 1024)
        if self.max_queue_size <= 0:
            raise ValueError("max_queue_size must be positive")
        self.engine = engine if engine is not None else LLMEngine(model, **kwargs)
        self.tokenizer = self.engine.tokenizer
        self.commands: Queue = Queue()
        self.handles: dict[int, Queue] = {}
        self._lock = Lock()
        self._counters = {k: 0 for k in ("requests_total", "requests_finished", "requests_cancelled",
                                         "requests_errors", "requests_rejected", "generated_tokens_total",
                                         "active_requests")}
        self.prometheus = PrometheusMetrics()
        self.thread = Thread(target=self._run, name="b200moe-engine", daemon=True)
        self.thread.start()

    # ------------------------------------------------------------- asyncio side
    async def add_request(self, prompt: str | list[int], sampling_params: SamplingParams) -> RequestHandle:
        with self._lock:
            active = self._counters["active_requests"]
        if active >= self.max_queue_size:
            self._reject()
            raise OverflowError("engine request queue is full")
        ack: Queue = Queue(maxsize=1)
        events: Queue = Queue()
        self.commands.put(("add", (prompt, sampling_params, events), ack))
        res = await asyncio.to_thread(ack.get)
        if isinstance(res, Exception):
            raise res
        return RequestHandle(res, events)

    async def next_event(self, handle: RequestHandle) -> TokenEvent:
        return await asyncio.to_thread(handle.events.get)

    def cancel(self, seq_id: int):
        self.commands.put(("cancel", (seq_id,), None))

    async def close(self):
        """Stop the engine thread and release the engine; later calls return at once."""
        if not self.thread.is_alive():
            return
        ack: Queue = Queue(maxsize=1)
        self.commands.put(("close", (), ack))
        while self.thread.is_alive():  # the thread may exit without answering (closed elsewhere)
            try:
                await asyncio.to_thread(ack.get, True, 0.5)
                break
            except Empty:
                continue
        await asyncio.to_thread(self.thread.join)

    def metrics(self) -> dict:
        with self._lock:
            m = dict(self._counters)
        m.update(self.engine.metrics())
        return m

    def prometheus_text(self) -> str:
        return self.prometheus.render(self.metrics())

    # ----------------------------------------------------------- engine thread
    def _bump(self, **d):
        with self._lock:
            for k, v in d.items():
                self._counters[k] += v

    def _reject(self):
        self._bump(requests_rejected=1)
        self.prometheus.rejected.inc()

    def _add(self, prompt, sp, events, ack):
        try:
            if len(self.handles) >= self.max_queue_size:
                self._reject()
                raise OverflowError("engine request queue is full")
            try:
                seq_id = self.engine.add_request(prompt, sp)
            except OverflowError:
                self._reject()
                raise
            self.handles[seq_id] = events
            self._bump(requests_total=1, active_requests=1)
            self.prometheus.requests.inc()
            self.prometheus.active.inc()
            ack.put(seq_id)
        except Exception as exc:
            ack.put(exc)

    def _cancel(self, seq_id):
        if self.engine.cancel_request(seq_id):
            ev = self.handles.pop(seq_id, None)
            if ev is not None:
                ev.put(TokenEvent(finished=True, cancelled=True))
            self._bump(requests_cancelled=1, active_requests=-1)
            self.prometheus.cancelled.inc()
            self.prometheus.active.dec()

    def _close(self, ack):
        n = len(self.handles)
        for seq_id, ev in list(self.handles.items()):
            self.engine.cancel_request(seq_id)
            ev.put(TokenEvent(finished=True, cancelled=True))
        self.handles.clear()
        if n:
            self._bump(requests_cancelled=n, active_requests=-n)
            self.prometheus.cancelled.inc(n)
            self.prometheus.active.set(0)
        try:
            self.engine.exit()
        finally:
            ack.put(True)

    def _handle(self, item) -> bool:
        cmd, args, ack = item
        if cmd == "add":
            self._add(*args, ack)
        elif cmd == "cancel":
            self._cancel(*args)
        elif cmd == "close":
            self._close(ack)
            return False
        return True

    def _fail_all(self, exc: BaseException):
        msg = f"{type(exc).__name__}: {exc}"
        n = len(self.handles)
        for seq_id, ev in list(self.handles.items()):
            ev.put(TokenEvent(finished=True, error=msg))
            try:
                self.engine.cancel_request(seq_id)
            except Exception:
                pass
        self.handles.clear()
        with self._lock:
            self._counters["active_requests"] = 0
            self._counters["requests_errors"] += n
        self.prometheus.errors.inc(n)
        self.prometheus.active.set(0)

    def _run(self):
        running = True
        while running:
            if self.engine.is_finished():
                try:
                    running = self._handle(self.commands.get(timeout=0.1))
                except Empty:
                    pass
                continue
            while running:
                try:
                    running = self._handle(self.commands.get_nowait())
                except Empty:
                    break
            if not running:
                break
            try:
                self.engine.step()
                step = self.engine.last_step_metrics or {}
                if step.get("mode") == "empty":
                    time.sleep(0.005)
                else:
                    self.prometheus.observe_step(step)
            except Exception as exc:
                self._fail_all(exc)
                continue
            for seq_id, tok, finished, metrics, lp in self.engine.last_token_events:
                ev = self.handles.get(seq_id)
                if ev is None:
                    continue
                ev.put(TokenEvent(token_id=tok, finished=finished, metrics=metrics, logprobs=lp))
                self._bump(generated_tokens_total=1)
                self.prometheus.generated_tokens.inc()
                if finished:
                    self.handles.pop(seq_id, None)
                    self._bump(requests_finished=1, active_requests=-1)
                    self.prometheus.finished.inc()
                    self.prometheus.active.dec()
                    self.prometheus.observe_request(metrics)
