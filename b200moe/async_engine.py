"""Online-serving front of :class:`LLMEngine`: asyncio callers on one side, one
engine thread on the other.

Threading model
  * The engine thread is the only thread that touches the ``LLMEngine``.  With
    nothing admitted it sleeps on a condition variable; otherwise it runs
    ``step()`` back to back (each step already overlaps host scheduling with the
    GPU through the engine's launch / collect pipeline).
  * Callers post to an inbox.  Admission (tokenise, length / vocabulary / KV
    checks) runs on the engine thread and answers through a
    ``concurrent.futures.Future`` that the caller awaits, so no thread is parked
    per request.
  * Tokens return through a per-request ``asyncio.Queue`` owned by the caller's
    event loop.  After a step the engine thread hands each loop ONE callback
    carrying that loop's events, so a waiting stream costs neither a thread nor
    a wake-up per token.

Contract kept from the reference server (nanovllm/async_engine.py): a request
queue that is full, or a request the KV pool can never hold, raises
``OverflowError`` (HTTP 429); an over-long or out-of-vocabulary request raises
``ValueError`` (HTTP 400); when a step raises, every in-flight request gets an
error event and the engine keeps serving; ``TokenEvent`` fields are what the
server reads; ``metrics()`` keys are the Prometheus service counters.
"""
from __future__ import annotations

import asyncio
import collections
import concurrent.futures
import threading
from dataclasses import dataclass

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
    """What ``add_request`` returns: the engine's sequence id and the request's event queue."""
    seq_id: int
    events: asyncio.Queue | None
    loop: asyncio.AbstractEventLoop | None = None


class _ServiceStats:
    """Service-level counters (the ``/metrics`` names), updated on the engine thread."""
    KEYS = ("requests_total", "requests_finished", "requests_cancelled", "requests_errors",
            "requests_rejected", "generated_tokens_total", "active_requests")
    __slots__ = KEYS + ("_lock",)

    def __init__(self):
        self._lock = threading.Lock()
        for k in self.KEYS:
            setattr(self, k, 0)

    def add(self, **delta):
        with self._lock:
            for k, v in delta.items():
                setattr(self, k, getattr(self, k) + v)

    def snapshot(self) -> dict:
        with self._lock:
            return {k: getattr(self, k) for k in self.KEYS}


class AsyncLLMEngine:

    def __init__(self, model: str | None = None, engine: LLMEngine | None = None, **kwargs):
        self.max_queue_size = kwargs.pop("max_queue_size", 1024)
        if self.max_queue_size <= 0:
            raise ValueError("max_queue_size must be positive")
        self.engine = engine if engine is not None else LLMEngine(model, **kwargs)
        self.tokenizer = self.engine.tokenizer
        self.stats = _ServiceStats()
        self.prometheus = PrometheusMetrics()
        self._cv = threading.Condition()
        self._inbox: collections.deque = collections.deque()
        self._pending_admits = 0                 # posted, not yet answered (guarded by _cv)
        self._streams: dict[int, RequestHandle] = {}   # engine thread only
        self._thread = threading.Thread(target=self._serve, name="b200moe-engine", daemon=True)
        self._thread.start()

    # ================================================================ callers
    async def add_request(self, prompt: str | list[int], sampling_params: SamplingParams) -> RequestHandle:
        loop = asyncio.get_running_loop()
        handle = RequestHandle(-1, asyncio.Queue(), loop)
        answer: concurrent.futures.Future = concurrent.futures.Future()
        with self._cv:
            full = self.stats.active_requests + self._pending_admits >= self.max_queue_size
            if not full:
                self._pending_admits += 1
                self._inbox.append(("admit", prompt, sampling_params, handle, answer))
                self._cv.notify()
        if full:
            self._count_rejection()
            raise OverflowError("engine request queue is full")
        handle.seq_id = await asyncio.wrap_future(answer)
        return handle

    async def next_event(self, handle: RequestHandle) -> TokenEvent:
        return await handle.events.get()

    def cancel(self, seq_id: int):
        self._post(("cancel", seq_id))

    async def close(self):
        """Cancel what is in flight, release the engine and stop the thread; later calls return at once."""
        if not self._thread.is_alive():
            return
        done: concurrent.futures.Future = concurrent.futures.Future()
        self._post(("close", done))
        while self._thread.is_alive() and not done.done():
            await asyncio.sleep(0.05)
        if done.done() and done.exception() is not None:
            raise done.exception()
        await asyncio.to_thread(self._thread.join)

    def metrics(self) -> dict:
        m = self.stats.snapshot()
        m.update(self.engine.metrics())
        return m

    def prometheus_text(self) -> str:
        return self.prometheus.render(self.metrics())

    def _post(self, cmd):
        with self._cv:
            self._inbox.append(cmd)
            self._cv.notify()

    def _count_rejection(self):
        self.stats.add(requests_rejected=1)
        self.prometheus.rejected.inc()

    # ========================================================== engine thread
    def _serve(self):
        while True:
            with self._cv:
                while not self._inbox and self.engine.is_finished():
                    self._cv.wait()
                commands = list(self._inbox)
                self._inbox.clear()
            for cmd in commands:
                if cmd[0] == "close":
                    self._shutdown(cmd[1])
                    return
                if cmd[0] == "admit":
                    self._admit(*cmd[1:])
                else:
                    self._drop(cmd[1], TokenEvent(finished=True, cancelled=True))
            if self.engine.is_finished():
                continue
            try:
                self.engine.step()
            except Exception as exc:  # a failed step fails its requests, not the server
                self._fail_in_flight(exc)
                continue
            self._deliver(self.engine.last_token_events)
            step = self.engine.last_step_metrics or {}
            if step.get("mode") == "empty":
                # nothing schedulable right now: wait briefly, or until a command arrives
                with self._cv:
                    if not self._inbox:
                        self._cv.wait(0.002)
            else:
                self.prometheus.observe_step(step)

    def _admit(self, prompt, sp, handle: RequestHandle, answer: concurrent.futures.Future):
        try:
            if len(self._streams) >= self.max_queue_size:
                raise OverflowError("engine request queue is full")
            seq_id = self.engine.add_request(prompt, sp)
        except Exception as exc:
            if isinstance(exc, OverflowError):
                self._count_rejection()
            with self._cv:
                self._pending_admits -= 1
            answer.set_exception(exc)
            return
        handle.seq_id = seq_id
        self._streams[seq_id] = handle
        with self._cv:  # active and pending move together, so the queue-full check never double counts
            self._pending_admits -= 1
            self.stats.add(requests_total=1, active_requests=1)
        self.prometheus.requests.inc()
        self.prometheus.active.inc()
        answer.set_result(seq_id)

    def _drop(self, seq_id: int, event: TokenEvent) -> bool:
        """Cancel ``seq_id`` in the engine and end its stream with ``event``; False if it was not live."""
        if not self.engine.cancel_request(seq_id):
            return False
        handle = self._streams.pop(seq_id, None)
        if handle is not None:
            self._send(handle.loop, [(handle.events, event)])
        self.stats.add(requests_cancelled=1, active_requests=-1)
        self.prometheus.cancelled.inc()
        self.prometheus.active.dec()
        return True

    def _deliver(self, events):
        """Route one step's ``(seq_id, token, finished, metrics, logprobs)`` events: one callback per loop."""
        per_loop: dict = {}
        tokens = finished = 0
        for seq_id, tok, done, metrics, lp in events:
            handle = self._streams.get(seq_id)
            if handle is None:
                continue
            per_loop.setdefault(handle.loop, []).append(
                (handle.events, TokenEvent(token_id=tok, finished=done, metrics=metrics, logprobs=lp)))
            tokens += 1
            if done:
                del self._streams[seq_id]
                finished += 1
                self.prometheus.observe_request(metrics)
        if tokens:
            self.stats.add(generated_tokens_total=tokens, requests_finished=finished, active_requests=-finished)
            self.prometheus.generated_tokens.inc(tokens)
            if finished:
                self.prometheus.finished.inc(finished)
                self.prometheus.active.dec(finished)
        for loop, items in per_loop.items():
            if not self._send(loop, items):
                for queue, _ in items:  # the caller's loop is gone: nobody will read these streams
                    gone = [sid for sid, h in self._streams.items() if h.events is queue]
                    for sid in gone:
                        self._drop(sid, TokenEvent(finished=True, cancelled=True))

    @staticmethod
    def _send(loop, items) -> bool:
        def put_all():
            for queue, ev in items:
                queue.put_nowait(ev)
        try:
            loop.call_soon_threadsafe(put_all)
            return True
        except RuntimeError:  # loop closed
            return False

    def _fail_in_flight(self, exc: BaseException):
        msg = f"{type(exc).__name__}: {exc}"
        streams, self._streams = self._streams, {}
        per_loop: dict = {}
        for seq_id, handle in streams.items():
            try:
                self.engine.cancel_request(seq_id)
            except Exception:
                pass
            per_loop.setdefault(handle.loop, []).append((handle.events, TokenEvent(finished=True, error=msg)))
        for loop, items in per_loop.items():
            self._send(loop, items)
        self.stats.add(requests_errors=len(streams), active_requests=-len(streams))
        self.prometheus.errors.inc(len(streams))
        self.prometheus.active.set(0)

    def _shutdown(self, done: concurrent.futures.Future):
        try:
            for seq_id in list(self._streams):
                if not self._drop(seq_id, TokenEvent(finished=True, cancelled=True)):
                    handle = self._streams.pop(seq_id)
                    self._send(handle.loop, [(handle.events, TokenEvent(finished=True, cancelled=True))])
                    self.stats.add(requests_cancelled=1, active_requests=-1)
            with self._cv:  # admissions that arrived with the close: refuse them
                rest = list(self._inbox)
                self._inbox.clear()
            for cmd in rest:
                if cmd[0] == "admit":
                    cmd[4].set_exception(OverflowError("engine is shutting down"))
            self.prometheus.active.set(0)
            self.engine.exit()
            done.set_result(True)
        except BaseException as exc:
            done.set_exception(exc)
