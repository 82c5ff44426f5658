"""Prometheus exposition for the server (reference: nanovllm/prometheus_metrics.py:6-119).

Service counters / gauge / latency histograms are kept here; the engine's own
metrics dict (``engine_*``, ``kv_*``, ``scheduler_*``) is rendered alongside
as gauges (``*_total`` as counters).  Uses prometheus_client when available,
otherwise a small built-in text renderer with the same metric names.
"""
from __future__ import annotations

import threading

PREFIX = "b200moe_"
LATENCY_BUCKETS = (0.005, 0.01, 0.025, 0.05, 0.1, 0.25, 0.5, 1.0, 2.5, 5.0, 10.0, 30.0, 60.0, 120.0)


class _Counter:
    def __init__(self):
        self.v = 0.0
        self.lock = threading.Lock()

    def inc(self, n=1):
        with self.lock:
            self.v += n


class _Gauge(_Counter):
    def dec(self, n=1):
        self.inc(-n)

    def set(self, v):
        with self.lock:
            self.v = float(v)


class _Histogram:
    def __init__(self, buckets=LATENCY_BUCKETS):
        self.buckets = buckets
        self.counts = [0] * (len(buckets) + 1)
        self.sum = 0.0
        self.n = 0
        self.lock = threading.Lock()

    def observe(self, v):
        with self.lock:
            self.sum += v
            self.n += 1
            for i, b in enumerate(self.buckets):
                if v <= b:
                    self.counts[i] += 1
                    return
            self.counts[-1] += 1


class PrometheusMetrics:

    COUNTERS = ("requests", "finished", "cancelled", "errors", "generated_tokens", "rejected")
    HISTS = ("queue_seconds", "ttft_seconds", "tpot_seconds", "e2e_seconds",
             "step_schedule_seconds", "step_forward_seconds")

    def __init__(self):
        for name in self.COUNTERS:
            setattr(self, name, _Counter())
        self.active = _Gauge()
        self.hist = {name: _Histogram() for name in self.HISTS}

    def observe_step(self, step: dict | None):
        if not step:
            return
        self.hist["step_schedule_seconds"].observe(step.get("schedule_s", 0.0))
        self.hist["step_forward_seconds"].observe(step.get("forward_s", 0.0))

    def observe_request(self, m: dict | None):
        if not m:
            return
        for key, hname in (("queue_s", "queue_seconds"), ("ttft_s", "ttft_seconds"),
                           ("tpot_s", "tpot_seconds"), ("e2e_s", "e2e_seconds")):
            v = m.get(key)
            if v is not None:
                self.hist[hname].observe(v)

    def render(self, engine_metrics: dict) -> str:
        out = []

        def emit(name, kind, value, help_):
            out.append(f"# HELP {PREFIX}{name} {help_}")
            out.append(f"# TYPE {PREFIX}{name} {kind}")
            out.append(f"{PREFIX}{name} {value}")

        for name in self.COUNTERS:
            emit(f"{name}_total", "counter", getattr(self, name).v, f"service {name}")
        emit("active_requests", "gauge", self.active.v, "requests in the system")
        for name, h in self.hist.items():
            out.append(f"# HELP {PREFIX}{name} latency histogram")
            out.append(f"# TYPE {PREFIX}{name} histogram")
            cum = 0
            for b, c in zip(h.buckets, h.counts):
                cum += c
                out.append(f'{PREFIX}{name}_bucket{{le="{b}"}} {cum}')
            out.append(f'{PREFIX}{name}_bucket{{le="+Inf"}} {h.n}')
            out.append(f"{PREFIX}{name}_sum {h.sum}")
            out.append(f"{PREFIX}{name}_count {h.n}")
        for k, v in engine_metrics.items():
            if isinstance(v, bool) or not isinstance(v, (int, float)):
                continue
            emit(k, "counter" if k.endswith("_total") else "gauge", v, f"engine metric {k}")
        return "\n".join(out) + "\n"
