"""Device-timed profiling ranges (reference: nanovllm/profiling.py:9-81).

``range(name, layer=None)`` records a pair of CUDA events around a region
(plain wall time on CPU) and, when NVTX is available, an NVTX range for
external profilers.  ``observe(name, value)`` records scalar observations.
``snapshot()`` synchronises once and returns per-range and per-layer
count / total / p50 / p95 in milliseconds.  Disabled profilers cost one
attribute check per range.
"""
from __future__ import annotations

import time
from collections import defaultdict
from contextlib import contextmanager

import torch


def percentile(values: list[float], q: float) -> float:
    if not values:
        return 0.0
    s = sorted(values)
    k = (len(s) - 1) * q / 100.0
    lo = int(k)
    hi = min(lo + 1, len(s) - 1)
    return s[lo] + (s[hi] - s[lo]) * (k - lo)


class DeviceProfiler:

    def __init__(self, device, enabled: bool = False):
        self.device = torch.device(device)
        self.enabled = enabled
        self._pending: list[tuple[str, int | None, object, object]] = []
        self._obs: dict[str, list[float]] = defaultdict(list)

    def start(self):
        self.enabled = True

    def stop(self):
        self.enabled = False

    @contextmanager
    def range(self, name: str, layer: int | None = None):
        if not self.enabled:
            yield
            return
        cuda = self.device.type == "cuda"
        if cuda:
            torch.cuda.nvtx.range_push(name)
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
        else:
            a = time.perf_counter()
        try:
            yield
        finally:
            if cuda:
                b.record()
                torch.cuda.nvtx.range_pop()
            else:
                b = time.perf_counter()
            self._pending.append((name, layer, a, b))

    def observe(self, name, value):
        """A scalar observation; a device tensor is read at ``snapshot()``
        (its one sync), not here."""
        if self.enabled:
            self._obs[name].append(value.detach() if isinstance(value, torch.Tensor) else float(value))

    def snapshot(self, reset: bool = True) -> dict:
        if self.device.type == "cuda" and self._pending:
            torch.cuda.synchronize(self.device)
        seg: dict[str, list[float]] = defaultdict(list)
        per_layer: dict[str, list[float]] = defaultdict(list)
        for name, layer, a, b in self._pending:
            ms = a.elapsed_time(b) if self.device.type == "cuda" else (b - a) * 1e3
            seg[name].append(ms)
            if layer is not None:
                per_layer[f"{name}@{layer}"].append(ms)

        def summ(d):
            return {k: {"count": len(v), "total_ms": sum(v), "p50_ms": percentile(v, 50),
                        "p95_ms": percentile(v, 95)} for k, v in d.items()}

        obs = {k: [float(x) for x in v] for k, v in self._obs.items()}
        out = {"segments": summ(seg), "layers": summ(per_layer),
               "observations": {k: {"count": len(v), "mean": sum(v) / len(v), "p50": percentile(v, 50),
                                    "p95": percentile(v, 95)} for k, v in obs.items() if v}}
        if reset:
            self._pending.clear()
            self._obs.clear()
        return out
