"""Metric definitions shared by the offline driver (``b200moe.bench_offline``),
the online client (``b200moe.bench_online``) and ``bench.py``.

Definitions follow the client-side serving convention the reference uses
(nanovllm/benchmarking.py:13-151), so numbers from either framework compare
directly:

* TTFT  request start -> first streamed token.
* TPOT  per request, (e2e - ttft) / (output_tokens - 1); ITL is the list of
        gaps between streamed outputs.
* percentiles default to nearest rank (index round((n-1) q)); ``linear``
  interpolates between order statistics (numpy's default).
* goodput counts requests meeting both SLOs per second; token goodput counts
  their output tokens; the strict SLO also bounds every inter-token gap.
* Wilson score interval for success proportions.
* failed requests fall into one of six buckets.
"""
from __future__ import annotations

import math
import statistics
from typing import Iterable, Sequence

ERROR_KINDS = ("none", "timeout", "http", "reject_429", "stream", "token_count")
Z95 = 1.959963984540054  # two-sided 95 % normal quantile


def _present(values: Iterable) -> list:
    return [v for v in values if v is not None]


def percentile(values: Iterable, q: float, method: str = "nearest"):
    """q in [0, 1]; None-valued entries are ignored; None when nothing is left."""
    if not 0.0 <= q <= 1.0:
        raise ValueError("percentile q must lie in [0, 1]")
    xs = sorted(_present(values))
    if not xs:
        return None
    pos = (len(xs) - 1) * q
    if method == "linear":
        lo = math.floor(pos)
        frac = pos - lo
        if frac == 0.0:
            return xs[lo]
        return xs[lo] + (xs[lo + 1] - xs[lo]) * frac
    if method != "nearest":
        raise ValueError(f"unknown percentile method {method!r}")
    return xs[min(len(xs) - 1, max(0, round(pos)))]


def request_tpot(e2e_s, ttft_s, output_tokens: int):
    """Time per output token after the first; None below two tokens."""
    if e2e_s is None or ttft_s is None or output_tokens < 2:
        return None
    return max(0.0, e2e_s - ttft_s) / (output_tokens - 1)


def coefficient_of_variation(values: Iterable) -> float:
    """Sample standard deviation / mean (0 for fewer than two samples)."""
    xs = list(values)
    if len(xs) < 2:
        return 0.0
    mu = statistics.fmean(xs)
    if mu == 0:
        return 0.0 if not any(xs) else math.inf
    return statistics.stdev(xs) / mu


def distribution(values: Iterable, prefix: str) -> dict:
    """{prefix}_p50_s / _p95_s / _p99_s (nearest rank)."""
    xs = _present(values)
    return {f"{prefix}_p{int(q * 100)}_s": percentile(xs, q) for q in (0.50, 0.95, 0.99)}


def _meets_slo(row: dict, ttft_slo_s: float, tpot_slo_s: float) -> bool:
    ttft, tpot = row.get("ttft_s"), row.get("tpot_s")
    return bool(row.get("ok")) and ttft is not None and tpot is not None and ttft <= ttft_slo_s \
        and tpot <= tpot_slo_s


def goodput(records: Sequence[dict], duration_s: float, ttft_slo_s: float, tpot_slo_s: float) -> float:
    """SLO-conforming requests per second."""
    if duration_s <= 0:
        return 0.0
    return sum(1 for r in records if _meets_slo(r, ttft_slo_s, tpot_slo_s)) / duration_s


def token_goodput(records: Sequence[dict], duration_s: float, conforming_key: str = "conforming_standard") -> float:
    """Output tokens of conforming requests per second."""
    if duration_s <= 0:
        return 0.0
    return sum((r.get("output_tokens") or 0) for r in records if r.get(conforming_key)) / duration_s


def wilson_ci(successes: int, total: int, z: float = Z95):
    """Wilson score interval (low, high) of successes / total; (None, None) if total == 0."""
    if total <= 0:
        return (None, None)
    p = successes / total
    zz_n = z * z / total
    denom = 1.0 + zz_n
    centre = (p + zz_n / 2.0) / denom
    half = z * math.sqrt(p * (1.0 - p) / total + zz_n / (4.0 * total)) / denom
    return (max(0.0, centre - half), min(1.0, centre + half))


def max_itl_s(row: dict):
    itls = row.get("itls_s") or []
    return max(itls) if itls else None


def classify_error(row: dict) -> str:
    """none / timeout / reject_429 / http / token_count / stream (everything else)."""
    if row.get("ok"):
        return "none"
    if row.get("timed_out"):
        return "timeout"
    status = row.get("http_status")
    if status is not None:
        return "reject_429" if status == 429 else "http"
    if "token usage missing" in (row.get("error") or ""):
        return "token_count"
    return "stream"


def error_bucket_counts(rows: Iterable[dict]) -> dict:
    counts = dict.fromkeys(ERROR_KINDS, 0)
    for r in rows:
        kind = classify_error(r)
        counts[kind] = counts.get(kind, 0) + 1
    return counts


def conforming(row: dict, ttft_slo_s: float, tpot_slo_s: float, strict_max_itl_s: float = 1.0):
    """(standard, strict): standard = both SLOs met; strict additionally needs
    every inter-token gap <= strict_max_itl_s (a request with no gaps passes)."""
    if not _meets_slo(row, ttft_slo_s, tpot_slo_s):
        return (False, False)
    return (True, all(g <= strict_max_itl_s for g in (row.get("itls_s") or [])))
