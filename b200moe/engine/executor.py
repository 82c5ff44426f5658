"""Runs engine steps on every rank.

One process per GPU.  Rank 0 lives in the engine's process; ranks 1..N-1 are
spawned workers, each owning its GPU and a :class:`ModelRunner`.  The control
plane is one duplex pipe per worker carrying small step plans (numpy arrays)
instead of pickled ``Sequence`` objects, with bounded waits on every reply:

* a worker that dies is seen as EOF on its pipe and raises :class:`RankFailure`
  on the driver at once;
* a worker that stops answering raises :class:`RankFailure` after
  ``rank_timeout_s``;
* a worker whose driver disappears exits on its own (parent-pid check).

Reference: the SharedMemory pickle channel + ``dist.barrier`` after every
command (nanovllm/engine/model_runner.py:168-246) and the exit watchdog
(llm_engine.py:134-177).
"""
from __future__ import annotations

import collections
import os
import socket
import time
import traceback

import numpy as np

from b200moe.config import Config
from b200moe.engine.step_plan import StepPlan, build_plan, empty_plan


class RankFailure(RuntimeError):
    """A worker rank died, hung past the limit, or raised."""


def free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _use_shm() -> bool:
    return os.environ.get("B200MOE_SHM_CHANNEL", "1") != "0"


def _worker_main(config: Config, rank: int, conn, parent_pid: int, shm_spec=None):
    if shm_spec is not None:
        from b200moe.engine.shm_channel import ShmLink
        conn = ShmLink(shm_spec[0], conn, 1, shm_spec[1])
    try:
        from b200moe.engine.model_runner import ModelRunner
        runner = ModelRunner(config, rank)
        conn.send(("ready", config.num_kvcache_blocks))
    except BaseException:
        try:
            conn.send(("error", traceback.format_exc()))
        finally:
            return
    failed_launches = 0
    while True:
        if not conn.poll(1.0):
            if os.getppid() != parent_pid:  # driver is gone: leave
                os._exit(1)
            continue
        try:
            cmd, args = conn.recv()
        except (EOFError, OSError):  # driver gone, or a frame failed its checks
            os._exit(1)
        if cmd == "exit":
            try:
                runner.exit()
            finally:
                conn.send(("ok", None))
            return
        if cmd == "launch":
            # enqueue the step and return to the pipe at once: the next plan can be
            # enqueued behind it before this one finishes (launch-ahead decode keeps
            # every rank's stream fed).  No reply on success; a failure is reported as
            # the step's reply, which the driver reads at its collect.
            try:
                runner.launch(*args)
            except BaseException:
                conn.send(("error", traceback.format_exc(), "run"))
                failed_launches += 1
            continue
        if cmd == "collect" and failed_launches:
            failed_launches -= 1  # that step's reply (its error) is already sent
            continue
        # replies carry their command's kind: a step's reply may still be
        # uncollected when the driver issues a call (KV offload under overlap)
        kind = "run" if cmd in ("run", "collect") else "call"
        try:
            res = getattr(runner, cmd)(*args)
            conn.send(("ok", res, kind))
        except BaseException:
            conn.send(("error", traceback.format_exc(), kind))


class Executor:

    def __init__(self, config: Config):
        self.config = config
        self.world = config.world_size
        self.dp = config.dp_size
        self.procs = []
        self.conns = []
        from b200moe.engine.model_runner import ModelRunner
        if self.world > 1:
            import multiprocessing as mp
            # The engine's process group is its own, even inside a torchrun job:
            # torchrun's agent-store flag would make every rank (rank 0 too) a
            # client of the engine's tcp:// rendezvous, with no server to reach.
            for var in ("TORCHELASTIC_USE_AGENT_STORE", "TORCHELASTIC_RESTART_COUNT"):
                os.environ.pop(var, None)
            if not config.distributed_init_method:
                config.distributed_init_method = f"tcp://127.0.0.1:{free_port()}"
            ctx = mp.get_context("spawn")
            for r in range(1, self.world):
                a, b = ctx.Pipe(duplex=True)
                spec = None
                if _use_shm():
                    # per-step messages go through shared memory; the pipe stays for
                    # wake-ups, oversize payloads and end-of-file on a dead peer
                    from b200moe.engine.shm_channel import ShmLink
                    a = ShmLink.create(a)
                    spec = a.spec()
                p = ctx.Process(target=_worker_main, args=(config, r, b, os.getpid(), spec), daemon=True)
                p.start()
                self.procs.append(p)
                self.conns.append(a)
        self.runner = ModelRunner(config, 0, self.world)
        for r, c in enumerate(self.conns, start=1):
            status, payload = self._recv(r, c, timeout=max(600.0, config.rank_timeout_s))
            if status != "ready":
                raise RankFailure(f"rank {r} failed to start:\n{payload}")
        self.runner._executor = self  # runner.call(...) reaches every rank
        self.max_blocks = self.runner.max_blocks
        self._inflight: collections.deque = collections.deque()  # (plans, rows) of launched steps
        # per worker, replies that arrived while another kind was awaited
        self._stash = [collections.deque() for _ in self.conns]

    # ------------------------------------------------------------ plumbing
    def _recv(self, rank: int, conn, timeout: float | None = None):
        timeout = self.config.rank_timeout_s if timeout is None else timeout
        deadline = time.monotonic() + timeout
        while True:
            remaining = deadline - time.monotonic()
            if remaining <= 0:
                raise RankFailure(f"rank {rank} did not answer within {timeout:.0f} s")
            try:
                if conn.poll(min(remaining, 1.0)):
                    return conn.recv()
            except (EOFError, OSError) as exc:
                raise RankFailure(f"rank {rank} exited ({exc!r})") from exc
            proc = self.procs[rank - 1]
            if not proc.is_alive():
                raise RankFailure(f"rank {rank} exited with code {proc.exitcode}")

    def _reply(self, rank: int, conn, kind: str, timeout: float | None = None):
        """The oldest reply of ``kind`` ("run" or "call") from ``rank``.  A
        worker answers in command order, so a call issued while steps are in
        flight first meets their replies: those wait in the stash, in order,
        for ``collect``."""
        stash = self._stash[rank - 1]
        for i, msg in enumerate(stash):
            if msg[2] == kind:
                del stash[i]
                return msg[0], msg[1]
        while True:
            msg = self._recv(rank, conn, timeout)
            if len(msg) < 3 or msg[2] == kind:
                return msg[0], msg[1]
            stash.append(msg)

    def _send_all(self, cmd: str, per_rank_args: list[tuple]):
        for r, c in enumerate(self.conns, start=1):
            try:
                c.send((cmd, per_rank_args[r]))
            except (BrokenPipeError, OSError) as exc:
                raise RankFailure(f"rank {r} is gone ({exc!r})") from exc

    def _gather(self, kind: str = "call") -> list:
        out = []
        for r, c in enumerate(self.conns, start=1):
            status, payload = self._reply(r, c, kind)
            if status != "ok":
                raise RankFailure(f"rank {r} raised:\n{payload}")
            out.append(payload)
        return out

    def call(self, method: str, *args):
        """Run ``runner.method(*args)`` on every rank; returns rank 0's result."""
        self._send_all(method, [args] * self.world)
        res = getattr(self.runner, method)(*args)
        self._gather()
        return res

    def call_all(self, method: str, *args) -> list:
        """Run ``runner.method(*args)`` on every rank; returns every rank's result."""
        self._send_all(method, [args] * self.world)
        res = getattr(self.runner, method)(*args)
        return [res] + self._gather()

    def call_rank(self, rank: int, method: str, *args):
        """Run ``runner.method(*args)`` on one rank only (its private KV pool)."""
        if rank == 0:
            return getattr(self.runner, method)(*args)
        c = self.conns[rank - 1]
        try:
            c.send((method, args))
        except (BrokenPipeError, OSError) as exc:
            raise RankFailure(f"rank {rank} is gone ({exc!r})") from exc
        status, payload = self._reply(rank, c, "call")
        if status != "ok":
            raise RankFailure(f"rank {rank} raised:\n{payload}")
        return payload

    def rank_caller(self, rank: int):
        """Object with ``call(method, *args)`` bound to one rank (KV offload hooks)."""
        ex = self

        class _Caller:
            def call(self, method, *args):
                return ex.call_rank(rank, method, *args)
        return _Caller()

    # --------------------------------------------------------------- steps
    def plans(self, batch, grammar_masks: dict | None = None, feed_from=None) -> list[StepPlan]:
        """One plan per rank: every row on every rank (tensor-parallel
        attention), or each sequence's rows on its data-parallel rank.
        ``feed_from``: the batch still in flight whose sampled tokens the decode
        rows of this batch read on the device (launch-ahead decode)."""
        seqs, q, flags = batch.sequences, batch.query_lens, batch.prefill_flags
        bs = self.config.kvcache_block_size
        feeds = self._feed_maps(feed_from) if feed_from is not None else [None] * self.world
        if self.dp == 1 and self.config.attention_parallel == "tp" and self.world > 1:
            plan = build_plan(seqs, q, flags, bs, self.max_blocks, feed=feeds[0])
            plans = [plan] * self.world  # tensor-parallel attention: every rank runs every row
        elif self.dp == 1:
            plans = [build_plan(seqs, q, flags, bs, self.max_blocks, feed=feeds[0])] + \
                    [empty_plan(self.max_blocks) for _ in range(self.world - 1)]
        else:
            parts: list[list[int]] = [[] for _ in range(self.world)]
            for i, s in enumerate(seqs):
                parts[max(s.dp_rank, 0)].append(i)
            plans = [build_plan([seqs[i] for i in idx], [q[i] for i in idx], [flags[i] for i in idx], bs,
                                self.max_blocks, rows=idx, feed=feeds[r]) if idx else empty_plan(self.max_blocks)
                     for r, idx in enumerate(parts)]
        if grammar_masks:
            for p in plans:
                g = [(r, grammar_masks[br]) for r, br in enumerate(p.rows.tolist()) if br in grammar_masks]
                if g:
                    p.grammar_rows = np.asarray([r for r, _ in g], np.int32)
                    p.grammar_mask = np.stack([m for _, m in g]).astype(np.int32)
        return plans

    def _feed_maps(self, batch) -> list[dict]:
        """Per rank, {id(sequence): plan row} of the newest launched step, which
        must be ``batch``: its rank-local sampled-token order."""
        plans, _ = self._inflight[-1]
        seqs = batch.sequences
        return [{id(seqs[br]): r for r, br in enumerate(p.rows.tolist())} for p in plans]

    def check_alive(self):
        for r, p in enumerate(self.procs, start=1):
            if not p.is_alive():
                raise RankFailure(f"rank {r} exited with code {p.exitcode}")

    def launch(self, batch, grammar_masks: dict | None = None, feed_from=None):
        plans = self.plans(batch, grammar_masks, feed_from)
        self.check_alive()
        self._send_all("launch", [(p,) for p in plans])
        try:
            self.runner.launch(plans[0])
        except RankFailure:
            raise
        except Exception as exc:
            # a collective that failed because a peer vanished or raised: report it
            for r, (p, c) in enumerate(zip(self.procs, self.conns), start=1):
                if not p.is_alive():
                    raise RankFailure(f"rank {r} exited with code {p.exitcode}") from exc
                try:
                    if c.poll(0):
                        status, payload = c.recv()[:2]
                        if status == "error":
                            raise RankFailure(f"rank {r} raised:\n{payload}") from exc
                except (EOFError, OSError):
                    raise RankFailure(f"rank {r} is gone") from exc
            if self.world > 1:
                # a collective timed out on a peer that neither exited nor reported
                # an error (hung): the rank group is out of step, fail the step
                raise RankFailure(f"collective failed with {self.world} ranks: {exc}") from exc
            raise
        self._inflight.append((plans, len(batch.sequences)))

    def collect(self):
        """Tokens (batch-row order) of the oldest launched step."""
        plans, n = self._inflight.popleft()
        self._send_all("collect", [()] * self.world)  # the workers wait on their own steps meanwhile
        results = [self.runner.collect()] + self._gather("run")
        tokens = [0] * n
        logprobs = None
        for plan, (toks, lps) in zip(plans, results):
            for r, t in zip(plan.rows.tolist(), toks):
                tokens[r] = t
            if lps is not None:
                logprobs = logprobs or [None] * n
                for r, lp in zip(plan.rows.tolist(), lps):
                    logprobs[r] = lp
        return tokens, logprobs

    def execute(self, batch):
        self.launch(batch)
        return self.collect()

    def exit(self):
        for r, c in enumerate(self.conns, start=1):
            try:
                if hasattr(c, "spec"):
                    c.send(("exit", ()), timeout=2.0)  # a hung peer never consumes: do not wait long
                else:
                    c.send(("exit", ()))
            except Exception:
                pass
        # this rank's teardown runs alongside the workers': releasing the peer-memory
        # buffers and destroying the process group are collectives every rank must reach,
        # so waiting for the workers' replies first would leave them blocked on rank 0
        if getattr(self, "runner", None) is not None:
            try:
                self.runner.exit()
            except Exception:
                pass  # the workers are still reaped below
            self.runner = None
        for r, c in enumerate(self.conns, start=1):
            try:
                self._recv(r, c, timeout=30.0)
            except Exception:
                pass
        for p in self.procs:
            p.join(timeout=10)
            if p.is_alive():
                p.kill()
        for c in self.conns:
            if hasattr(c, "close") and hasattr(c, "spec"):
                c.close()
        self.procs, self.conns = [], []
        if getattr(self, "runner", None) is not None:
            self.runner.exit()
            self.runner = None
