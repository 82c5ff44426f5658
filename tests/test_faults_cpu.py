"""Failure detection on the host (no GPU is ever faulted): a worker rank that
dies or stops answering is detected within the bound and surfaces as
RankFailure; an engine step exception fails every in-flight request and the
server keeps serving; the exit watchdog bounds a wedged teardown."""
import asyncio
import os
import signal
import subprocess
import sys
import textwrap
import time

import pytest

from b200moe import LLM, SamplingParams
from b200moe.async_engine import AsyncLLMEngine
from b200moe.engine.executor import RankFailure

KW = dict(device="cpu", kvcache_block_size=16, num_kvcache_blocks=64, max_num_batched_tokens=256,
          max_num_seqs=8, max_model_len=256, enforce_eager=True)
SP = SamplingParams(temperature=0.0, max_tokens=4, ignore_eos=True)


def test_dead_worker_detected():
    llm = LLM("tiny-moe", tensor_parallel_size=2, rank_timeout_s=20, **KW)
    try:
        assert llm.generate([[1, 2, 3]], SP, use_tqdm=False)[0]["token_ids"]
        proc = llm.executor.procs[0]
        os.kill(proc.pid, signal.SIGKILL)
        proc.join(5)
        t0 = time.monotonic()
        with pytest.raises(RankFailure):
            llm.generate([[4, 5, 6]], SP, use_tqdm=False)
        assert time.monotonic() - t0 < 20
    finally:
        llm.exit()


def test_hung_worker_times_out():
    # the limit also bounds the ranks' start-up rendezvous: leave room for a cold import
    llm = LLM("tiny-moe", tensor_parallel_size=2, rank_timeout_s=20, **KW)
    try:
        proc = llm.executor.procs[0]
        os.kill(proc.pid, signal.SIGSTOP)  # alive but never answers
        t0 = time.monotonic()
        with pytest.raises(RankFailure):
            llm.generate([[4, 5, 6]], SP, use_tqdm=False)
        assert time.monotonic() - t0 < 60
        os.kill(proc.pid, signal.SIGKILL)
    finally:
        llm.exit()


def test_step_exception_fails_requests_and_engine_keeps_serving():
    eng = AsyncLLMEngine("tiny-moe", **KW)
    try:
        real_step = eng.engine.step
        calls = {"n": 0}

        def flaky():
            calls["n"] += 1
            if calls["n"] == 1:
                raise RuntimeError("injected step failure")
            return real_step()

        eng.engine.step = flaky

        async def one():
            h = await eng.add_request([1, 2, 3, 4], SP)
            toks, err = [], None
            while True:
                ev = await eng.next_event(h)
                if ev.error:
                    err = ev.error
                    break
                if ev.token_id is not None:
                    toks.append(ev.token_id)
                if ev.finished:
                    break
            return toks, err

        _, err = asyncio.run(one())
        assert err and "injected step failure" in err
        toks, err = asyncio.run(one())  # the engine thread survived
        assert err is None and len(toks) == 4
        assert eng.metrics()["requests_errors"] >= 1
    finally:
        asyncio.run(eng.close())


def test_exit_watchdog_bounds_wedged_teardown(tmp_path):
    """A teardown that never returns is killed by the watchdog (runs in a child)."""
    code = textwrap.dedent("""
        import os, sys, time
        sys.path.insert(0, %r)
        os.environ["B200MOE_EXIT_TIMEOUT_S"] = "2"
        from b200moe.engine.llm_engine import LLMEngine
        eng = LLMEngine.__new__(LLMEngine)
        eng._exited = False
        class Wedged:
            procs = []
            def exit(self):
                time.sleep(3600)
        eng.executor = Wedged()
        eng.exit()
        print("unreachable")
    """ % os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    for rc in ("0", "5"):  # the forced exit's status is configurable (tests use a non-zero one)
        t0 = time.monotonic()
        r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=60,
                           env={**os.environ, "B200MOE_EXIT_WATCHDOG_RC": rc})
        assert time.monotonic() - t0 < 30
        assert "unreachable" not in r.stdout
        assert "watchdog" in r.stderr
        assert r.returncode == int(rc), (r.returncode, r.stderr[-300:])


def _link_pair(capacity=1 << 16):
    import multiprocessing as mp
    from b200moe.engine.shm_channel import ShmLink
    a, b = mp.Pipe(duplex=True)
    drv = ShmLink.create(a, capacity=capacity)
    wrk = ShmLink(drv.spec()[0], b, 1, capacity)
    return drv, wrk


def test_control_frame_checks_reject_torn_and_stale_messages():
    from b200moe.engine import shm_channel as sc
    drv, wrk = _link_pair()
    try:
        drv.send(("step", [1, 2, 3]))
        assert wrk.recv() == ("step", [1, 2, 3])
        wrk.send(("ok", 7))
        assert drv.recv() == ("ok", 7)
        # a flipped byte in the body fails the checksum
        drv.send(("step", list(range(100))))
        with wrk._region(0) as region:
            region[sc.HEADER.size + 20] ^= 0xFF
        with pytest.raises(sc.ControlMessageError, match="checksum"):
            wrk.recv()
    finally:
        wrk.close()
        drv.close()
    drv, wrk = _link_pair()
    try:
        drv.send(("a", 1))
        # a frame stamped with another sequence number (a stale or replayed plan)
        with wrk._region(0) as region:
            sc.HEADER.pack_into(region, 0, 5, 0)
        with pytest.raises(sc.ControlMessageError, match="sequence 5, expected 1"):
            wrk.recv()
    finally:
        wrk.close()
        drv.close()


def test_oversize_frames_travel_on_the_pipe_and_are_checked():
    from b200moe.engine import shm_channel as sc
    drv, wrk = _link_pair(capacity=4096)
    try:
        big = bytes(range(256)) * 64
        drv.send(("big", big))
        assert wrk.recv() == ("big", big)
        wrk.send(("ok", None))
        assert drv.recv() == ("ok", None)
    finally:
        wrk.close()
        drv.close()
    assert issubclass(sc.ControlMessageError, OSError)  # the executor's liveness path catches OSError


def test_corrupt_step_plan_fails_the_rank_not_the_model(monkeypatch):
    """The driver's frames to rank 1 go out with a wrong checksum: the worker
    rejects the frame and leaves, and the driver reports RankFailure within
    the rank timeout instead of running a torn step."""
    from b200moe.engine import shm_channel as sc
    llm = LLM("tiny-moe", tensor_parallel_size=2, rank_timeout_s=20, **KW)
    try:
        assert llm.generate([[1, 2, 3]], SP, use_tqdm=False)[0]["token_ids"]
        real = sc.frame
        monkeypatch.setattr(sc, "frame", lambda seq, body: real(seq, body[:-1] + bytes([body[-1] ^ 1])))
        t0 = time.monotonic()
        with pytest.raises(RankFailure):
            llm.generate([[4, 5, 6]], SP, use_tqdm=False)
        assert time.monotonic() - t0 < 20
        monkeypatch.setattr(sc, "frame", real)
    finally:
        llm.exit()


def test_worker_killed_mid_generate_fails_within_bound():
    """A rank killed while steps are running (rank 0 may be inside a collective
    with it): the driver raises RankFailure within the process-group timeout
    instead of waiting for good."""
    import threading
    llm = LLM("tiny-moe", tensor_parallel_size=2, rank_timeout_s=20, **KW)
    try:
        proc = llm.executor.procs[0]
        threading.Timer(1.0, lambda: os.kill(proc.pid, signal.SIGKILL)).start()
        long = SamplingParams(temperature=0.0, max_tokens=200, ignore_eos=True)
        t0 = time.monotonic()
        with pytest.raises(RankFailure):
            for _ in range(50):  # keeps stepping until the kill lands
                llm.generate([[1, 2, 3, 4]] * 4, long, use_tqdm=False)
        assert time.monotonic() - t0 < 60
    finally:
        llm.exit()


def test_driver_tears_down_alongside_workers():
    """Rank 0 releases its own collective resources (peer-memory buffers, process
    group) after telling the workers to exit and before waiting for their replies:
    a worker's teardown waits in those collectives for rank 0."""
    from b200moe.engine.executor import Executor
    order = []

    class Runner:
        def exit(self):
            order.append("runner")

    class Conn:
        def send(self, msg, timeout=None):
            order.append("send")

    ex = Executor.__new__(Executor)
    ex.runner, ex.conns, ex.procs = Runner(), [Conn(), Conn()], []

    def recv(r, c, timeout):
        assert "runner" in order, "a worker's exit reply needs rank 0's collectives first"
        order.append("recv")

    ex._recv = recv
    ex.exit()
    assert order == ["send", "send", "runner", "recv", "recv"]
