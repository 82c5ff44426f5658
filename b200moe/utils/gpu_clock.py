"""Samples SM clocks and throttle reasons with ``nvidia-smi`` during a timed region.

Read-only: it queries clocks, it never sets them.
"""
from __future__ import annotations

import csv
import os
import shutil
import statistics
import subprocess
import tempfile

QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


class ClockSampler:

    def __init__(self, gpus: list[int] | None = None, period_ms: int = 200):
        self.gpus = gpus
        self.period_ms = period_ms
        self.proc = None
        self.path = None

    def __enter__(self):
        if shutil.which("nvidia-smi") is None:
            return self
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        cmd = ["nvidia-smi", f"--query-gpu={QUERY}", "--format=csv,noheader,nounits", "-lms", str(self.period_ms)]
        if self.gpus is not None:
            cmd += ["-i", ",".join(str(g) for g in self.gpus)]
        self.proc = subprocess.Popen(cmd, stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        if not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        with open(self.path) as f:
            for r in csv.reader(f):
                if len(r) >= 9:
                    rows.append([c.strip() for c in r])
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None

        sm = [num(r[1]) for r in rows if num(r[1]) is not None]
        smax = [num(r[2]) for r in rows if num(r[2]) is not None]
        loaded = [s for s in sm if s > 0.5 * (max(sm) if sm else 1)] or sm
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": max(smax) if smax else None, "reasons": reasons, "samples": len(rows)}
