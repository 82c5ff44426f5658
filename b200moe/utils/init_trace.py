"""Per-rank initialisation milestones (reference: nanovllm/engine/model_runner.py:28, 82-92
prints per-stage init timings under ``NANOVLLM_TRACE_INIT``; nanovllm/entrypoints/api_server.py:669-672
arms ``faulthandler.dump_traceback_later(180)``).

Every stage of a rank's start-up (device, process group, model build, weights,
workspace, KV pool, graph capture) is timed and kept in ``stages``.  With
``B200MOE_TRACE_INIT=1`` each milestone is also printed as it is reached, and a
``faulthandler`` watchdog dumps every thread's stack if start-up has not
finished after ``B200MOE_TRACE_INIT_DUMP_S`` seconds (default 180), so a rank
stuck in a rendezvous or a capture shows where it is without being killed.
"""
from __future__ import annotations

import faulthandler
import os
import sys
import time


def enabled() -> bool:
    return os.environ.get("B200MOE_TRACE_INIT", "0") not in ("", "0")


class InitTrace:

    def __init__(self, rank: int):
        self.rank = rank
        self.verbose = enabled()
        self.t0 = self.last = time.perf_counter()
        self.stages: dict[str, float] = {}
        self._armed = False
        if self.verbose:
            limit = float(os.environ.get("B200MOE_TRACE_INIT_DUMP_S", "180"))
            if limit > 0:
                faulthandler.dump_traceback_later(limit, repeat=False, file=sys.stderr, exit=False)
                self._armed = True

    def mark(self, stage: str) -> None:
        now = time.perf_counter()
        self.stages[stage] = self.stages.get(stage, 0.0) + (now - self.last)
        self.last = now
        if self.verbose:
            print(f"[init] rank {self.rank} {stage} +{self.stages[stage]:.3f}s (total {now - self.t0:.3f}s)",
                  flush=True)

    def done(self) -> dict[str, float]:
        if self._armed:
            faulthandler.cancel_dump_traceback_later()
            self._armed = False
        self.stages["total"] = time.perf_counter() - self.t0
        if self.verbose:
            print(f"[init] rank {self.rank} ready in {self.stages['total']:.3f}s", flush=True)
        return self.stages
