"""Online serving benchmark: an HTTP streaming client against the OpenAI server.

    python -m b200moe.bench_online --base-url http://127.0.0.1:8000 --model m \
        --mode poisson --max-qps 4 --fractions 0.25,0.5,1 --requests 128 --output online.json
    python -m b200moe.bench_online ... --concurrency 8,32,128 --duration 60

Behaviour follows the reference's client (scripts/benchmark_online.py:39-893,
output schema version 3):

* **Load.** ``poisson``: open-loop arrivals at ``max_qps * fraction`` (exponential
  or ``fixed`` gaps, seeded).  ``concurrency``: each of N workers sends its next
  request when the previous one ends (``--duration`` stops submission).
* **Prompts.** ``shared`` repeats one word (prefix-cache friendly), ``unique``
  changes every word per request (no full-block reuse), ``mixed`` sends a
  3:4:3 short / medium / long mix.  ``--prompt-tokens`` calibrates word counts
  to a token target with ``--tokenizer``; ``--prompt-seed-per-repeat`` keeps
  repeats cold.
* **Token-id prompts.** ``--prompt-dist lognormal`` sends random token ids
  (below ``--prompt-vocab``) to ``/v1/completions`` with lognormal lengths
  (``--prompt-median``, ``--prompt-sigma``, clipped to ``--prompt-min`` /
  ``--prompt-max``); ``--output-len-range LO,HI`` draws each request's
  ``max_tokens`` uniformly (with ``ignore_eos``); ``--temperature`` / ``--top-p``
  set the sampling; ``--max-concurrency`` caps in-flight Poisson requests
  (a request waits for a slot and is timed from when it is sent).
  ``--workload online`` presets all of these to the headline online shape:
  lognormal median 1500 in [128, 8192], outputs 64..512, T 0.7, top-p 0.9,
  at most 64 in flight.
* **Per request** (streamed ``/v1/chat/completions``, or ``/v1/completions``
  for token-id prompts, with usage and server metrics): TTFT, ITLs, TPOT, e2e, token counts, ``[DONE]`` seen, HTTP status,
  timeout, error bucket.
* **Per point**: throughput, goodput (requests and tokens), standard / strict
  SLO rates with Wilson intervals, admission counts (429s), latency
  distributions, prefix-cache hit rate and engine step counts from a
  ``/metrics`` scrape before and after, GPU memory / utilisation maxima from
  ``nvidia-smi`` sampled during the point.
* **Aggregate** over repeats: pooled SLO rates with Wilson intervals.
"""
from __future__ import annotations

import argparse
import asyncio
import itertools
import json
import random
import subprocess
import threading
import time
from pathlib import Path

from b200moe.benchmarking import (classify_error, coefficient_of_variation, conforming, distribution,
                                  error_bucket_counts, percentile, request_tpot, token_goodput, wilson_ci)

SCHEMA_VERSION = 3
# named workloads; explicit flags override them
WORKLOADS = {
    # Poisson arrivals, at most 64 in flight; lognormal prompts of random token ids
    # (median 1500, clipped to [128, 8192]); outputs uniform in [64, 512]; T 0.7, top-p 0.9
    "online": dict(mode="poisson", prompt_dist="lognormal", prompt_median=1500.0, prompt_min=128, prompt_max=8192,
                   output_len_range=(64, 512), temperature=0.7, top_p=0.9, max_concurrency=64),
}
METRIC_PREFIX = "b200moe_"
PROMPT_SEED_STRIDE = 1_000_003


# ------------------------------------------------------------------ helpers
async def scrape_metrics(client, base_url: str) -> dict:
    """Unlabelled ``b200moe_*`` samples of ``/metrics`` as {name_without_prefix: value}."""
    try:
        r = await client.get(f"{base_url.rstrip('/')}/metrics", timeout=10.0)
        r.raise_for_status()
    except Exception as exc:  # noqa: BLE001 - reported in the payload
        return {"error": f"{type(exc).__name__}: {exc}"}
    out = {}
    for line in r.text.splitlines():
        if not line or line[0] == "#":
            continue
        name, _, value = line.strip().partition(" ")
        if name.startswith(METRIC_PREFIX) and "{" not in name:
            try:
                out[name[len(METRIC_PREFIX):]] = float(value)
            except ValueError:
                pass
    return out


def metrics_delta(before: dict, after: dict) -> dict:
    return {k: v - before.get(k, 0.0) for k, v in after.items()
            if isinstance(v, (int, float)) and isinstance(before.get(k, 0.0), (int, float))}


class ConcurrencyTracker:
    def __init__(self):
        self.current = self.maximum = 0

    def enter(self):
        self.current += 1
        self.maximum = max(self.maximum, self.current)

    def exit(self):
        self.current -= 1


class GpuSampler:
    """``nvidia-smi`` utilisation / memory on a background thread (read-only queries)."""

    def __init__(self, interval_s: float = 2.0, enabled: bool = True):
        self.interval_s, self.enabled = interval_s, enabled
        self.samples: list[dict] = []
        self.phase = "idle"
        self._stop = threading.Event()
        self._thread = None

    def start(self):
        if self.enabled:
            self._thread = threading.Thread(target=self._loop, daemon=True)
            self._thread.start()

    def _loop(self):
        while not self._stop.is_set():
            s = {"ts": time.perf_counter(), "phase": self.phase, "gpus": []}
            try:
                out = subprocess.run(["nvidia-smi", "--query-gpu=index,utilization.gpu,memory.used,memory.total",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True,
                                     timeout=15).stdout
                for line in out.strip().splitlines():
                    i, u, m, t = (x.strip() for x in line.split(","))
                    s["gpus"].append({"id": int(i), "util_pct": int(u), "mem_mib": int(m), "mem_total_mib": int(t)})
            except Exception as exc:  # noqa: BLE001
                s["error"] = f"{type(exc).__name__}: {exc}"
            self.samples.append(s)
            self._stop.wait(self.interval_s)

    def max_for(self, phase: str):
        per: dict[int, dict] = {}
        for s in self.samples:
            if s["phase"] != phase:
                continue
            for g in s["gpus"]:
                e = per.setdefault(g["id"], {"mem_mib": 0, "util_pct": 0})
                e["mem_mib"] = max(e["mem_mib"], g["mem_mib"])
                e["util_pct"] = max(e["util_pct"], g["util_pct"])
        return [per[k] for k in sorted(per)] or None

    def stop(self):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=20)


def mixed_bucket(request_id: int) -> str:
    slot = request_id % 10
    return "short" if slot < 3 else "medium" if slot < 7 else "long"


def build_prompt(word: str, n_words: int, mode: str, seed: int, request_id: int) -> str:
    if mode == "shared":
        return (word + " ") * n_words
    if mode == "unique":
        return " ".join(f"{word}-{seed}-{request_id}-{i}" for i in range(n_words))
    raise ValueError(f"unsupported prompt mode {mode!r}")


def repeat_prompt_seed(base: int, repeat: int, per_repeat: bool) -> int:
    return base if not per_repeat else base + (repeat - 1) * PROMPT_SEED_STRIDE


def token_count(tokenizer, text: str):
    if tokenizer is None:
        return None
    return len(tokenizer.encode(text))


def calibrate_words(tokenizer, word: str, mode: str, seed: int, target: int, iters: int = 8):
    """(words, tokens) whose prompt tokenises within 1 % (or 8 tokens) of ``target``."""
    words, best = max(8, target // 4), None
    for _ in range(iters):
        n = token_count(tokenizer, build_prompt(word, words, mode, seed, 0))
        if best is None or abs(n - target) < abs(best[1] - target):
            best = (words, n)
        if abs(n - target) <= max(8, target // 100):
            break
        words = max(1, round(words * target / max(n, 1)))
    return best


def arrival_offsets(count: int, qps: float, pattern: str, seed: int) -> list[float]:
    if pattern == "fixed":
        return [i / qps for i in range(count)]
    rng, t, out = random.Random(seed), 0.0, []
    for _ in range(count):
        out.append(t)
        t += rng.expovariate(qps)
    return out


# ------------------------------------------------------------------ requests
class RequestShape:
    """Endpoint, sampling fields and per-request output length of a run."""

    def __init__(self, args=None):
        self.temperature = getattr(args, "temperature", 0.0)
        self.top_p = getattr(args, "top_p", 1.0)
        self.token_prompts = getattr(args, "prompt_dist", "words") == "lognormal"
        self.out_range = getattr(args, "output_len_range", None)
        self.seed = getattr(args, "seed", 0)
        self.semaphore = None
        if getattr(args, "max_concurrency", 0):
            self.semaphore = asyncio.Semaphore(args.max_concurrency)

    def max_tokens(self, default: int, request_id: int) -> int:
        if not self.out_range:
            return default
        lo, hi = self.out_range
        return random.Random(self.seed * 7919 + request_id).randint(lo, hi)

    def body(self, model, prompt, max_tokens, include_metrics) -> dict:
        b = {"model": model, "temperature": self.temperature, "max_tokens": max_tokens, "stream": True,
             "stream_options": {"include_usage": True, "include_metrics": include_metrics}}
        if self.top_p < 1.0:
            b["top_p"] = self.top_p
        if self.out_range:
            b["ignore_eos"] = True  # the drawn length is the output length
        if self.token_prompts:
            b["prompt"] = prompt
        else:
            b["messages"] = [{"role": "user", "content": prompt}]
        return b


def lognormal_prompt(seed: int, request_id: int, median: float, sigma: float, lo: int, hi: int,
                     vocab: int) -> list[int]:
    """Random token ids; length lognormal(ln median, sigma) clipped to [lo, hi]."""
    import math
    rng = random.Random(seed * PROMPT_SEED_STRIDE + request_id)
    n = int(round(rng.lognormvariate(math.log(median), sigma)))
    n = max(lo, min(hi, n))
    return [rng.randrange(vocab) for _ in range(n)]


async def one_request(client, url, model, prompt, max_tokens, request_id, due, tracker, tokenizer=None,
                      request_timeout_s=None, include_metrics=True, shape: RequestShape | None = None) -> dict:
    shape = shape or RequestShape()
    await asyncio.sleep(max(0.0, due - time.perf_counter()))
    if shape.semaphore is not None:
        await shape.semaphore.acquire()
    try:
        return await _one_request(client, url, model, prompt, shape.max_tokens(max_tokens, request_id), request_id,
                                  due, tracker, tokenizer, request_timeout_s, include_metrics, shape)
    finally:
        if shape.semaphore is not None:
            shape.semaphore.release()


async def _one_request(client, url, model, prompt, max_tokens, request_id, due, tracker, tokenizer,
                       request_timeout_s, include_metrics, shape) -> dict:
    start = time.perf_counter()
    tracker.enter()
    st = {"first": None, "done": False, "usage": None, "finish": None, "server": None, "text": "", "status": None}
    times: list[float] = []
    error, timed_out = None, False
    body = shape.body(model, prompt, max_tokens, include_metrics)

    async def consume():
        async with client.stream("POST", url, json=body, timeout=None) as resp:
            st["status"] = resp.status_code
            resp.raise_for_status()
            async for line in resp.aiter_lines():
                if not line.startswith("data: "):
                    continue
                if line == "data: [DONE]":
                    st["done"] = True
                    continue
                ev = json.loads(line[6:])
                st["usage"] = ev.get("usage") or st["usage"]
                st["server"] = ev.get("metrics") or st["server"]
                choices = ev.get("choices") or []
                if not choices:
                    continue
                st["finish"] = choices[0].get("finish_reason") or st["finish"]
                content = (choices[0].get("delta") or {}).get("content") if "delta" in choices[0] \
                    else choices[0].get("text")
                if content:
                    now = time.perf_counter()
                    st["text"] += content
                    times.append(now)
                    if st["first"] is None:
                        st["first"] = now

    try:
        if request_timeout_s:
            await asyncio.wait_for(consume(), timeout=request_timeout_s)
        else:
            await consume()
    except asyncio.TimeoutError:
        error, timed_out = f"request timeout after {request_timeout_s}s", True
    except Exception as exc:  # noqa: BLE001 - bucketed below
        error = f"{type(exc).__name__}: {exc}"
        resp = getattr(exc, "response", None)
        if resp is not None:
            st["status"] = getattr(resp, "status_code", st["status"])
    finally:
        end = time.perf_counter()
        tracker.exit()
    usage = st["usage"]
    prompt_tokens = usage.get("prompt_tokens") if usage else (
        len(prompt) if isinstance(prompt, list) else token_count(tokenizer, prompt))
    output_tokens = usage.get("completion_tokens") if usage else token_count(tokenizer, st["text"])
    if error is None and not st["done"]:
        error = "stream ended before [DONE]"
    if error is None and (prompt_tokens is None or output_tokens is None):
        error = "token usage missing and no local tokenizer was configured"
    ttft = None if st["first"] is None else st["first"] - start
    row = {"request_id": request_id, "scheduled_s": due, "started_s": start, "arrival_lag_s": start - due,
           "ended_s": end, "e2e_s": end - start, "ttft_s": ttft,
           "tpot_s": request_tpot(end - start, ttft, output_tokens or 0),
           "itls_s": [b - a for a, b in zip(times, times[1:])], "prompt_tokens": prompt_tokens,
           "output_tokens": output_tokens, "stream_events": len(times), "done_received": st["done"],
           "finish_reason": st["finish"], "ok": error is None, "error": error, "timed_out": timed_out,
           "http_status": st["status"]}
    srv = st["server"]
    if srv:
        for k in ("queue_s", "ttft_s", "e2e_s", "tpot_s"):
            row[f"server_{k}"] = srv.get(k)
    row["error_kind"] = classify_error(row)
    return row


def _url(args) -> str:
    route = "completions" if getattr(args, "prompt_dist", "words") == "lognormal" else "chat/completions"
    return f"{args.base_url.rstrip('/')}/v1/{route}"


async def warmup(client, args, prompt_for, tokenizer, point_index):
    if args.warmup_requests <= 0:
        return
    tr, t0 = ConcurrencyTracker(), time.perf_counter() + 0.05
    rows = await asyncio.gather(*[
        one_request(client, _url(args), args.model, prompt_for(-1 - point_index * args.warmup_requests - i),
                    args.max_tokens, -i - 1, t0 + i * 0.05, tr, tokenizer, args.request_timeout_s,
                    shape=args.shape)
        for i in range(args.warmup_requests)])
    bad = [r for r in rows if not r["ok"]]
    if bad:
        raise RuntimeError(f"warmup failed: {bad[0]['error']}")


async def run_point_poisson(client, args, fraction, point_index, repeat, prompt_for, tokenizer):
    qps = args.max_qps * fraction
    await warmup(client, args, prompt_for, tokenizer, point_index)
    before = await scrape_metrics(client, args.base_url)
    t0 = time.perf_counter() + 0.2
    offs = arrival_offsets(args.requests, qps, args.arrival_pattern, args.seed + point_index)
    tr = ConcurrencyTracker()
    rows = await asyncio.gather(*[
        one_request(client, _url(args), args.model, prompt_for(point_index * args.requests + i), args.max_tokens, i,
                    t0 + offs[i], tr, tokenizer, args.request_timeout_s, shape=args.shape)
        for i in range(args.requests)])
    after = await scrape_metrics(client, args.base_url)
    for r in rows:
        r.update({"load_fraction": fraction, "target_qps": qps, "repeat": repeat})
    return list(rows), before, after, tr.maximum


async def run_point_concurrency(client, args, concurrency, point_index, repeat, prompt_for, tokenizer):
    concurrency = int(concurrency)
    await warmup(client, args, prompt_for, tokenizer, point_index)
    before = await scrape_metrics(client, args.base_url)
    t0 = time.perf_counter() + 0.2
    deadline = t0 + args.duration if args.duration else None
    tr, rows, ids = ConcurrencyTracker(), [], itertools.count()

    async def worker():
        for i in ids:
            if i >= args.requests or (deadline is not None and time.perf_counter() > deadline):
                return
            r = await one_request(client, _url(args), args.model, prompt_for(point_index * args.requests + i),
                                  args.max_tokens, i, t0, tr, tokenizer, args.request_timeout_s, shape=args.shape)
            r.update({"concurrency": concurrency, "repeat": repeat})
            rows.append(r)

    await asyncio.gather(*[worker() for _ in range(min(concurrency, args.requests))])
    after = await scrape_metrics(client, args.base_url)
    return rows, before, after, tr.maximum


# ------------------------------------------------------------------ summaries
def admission_summary(rows: list[dict]) -> dict:
    admitted = [r for r in rows if r.get("http_status") is not None and 200 <= r["http_status"] < 300]
    n, rej = len(admitted), sum(r.get("http_status") == 429 for r in rows)
    std = sum(bool(r.get("conforming_standard")) for r in admitted)
    strict = sum(bool(r.get("conforming_strict")) for r in admitted)
    return {"admission_counts": {"admitted": n, "reject_429": rej,
                                 "unknown": sum(r.get("http_status") is None for r in rows),
                                 "other_http": sum(r.get("http_status") is not None and r["http_status"] != 429
                                                   and not 200 <= r["http_status"] < 300 for r in rows),
                                 "conforming_standard": std, "conforming_strict": strict},
            "reject_429_rate": rej / len(rows) if rows else None,
            "admitted_slo_standard_rate": std / n if n else None,
            "admitted_slo_strict_rate": strict / n if n else None}


def summarize(rows: list[dict], max_conc: int, delta: dict, args, label: dict, gpu_max=None) -> dict:
    if not rows:
        raise ValueError("benchmark point produced no requests")
    good = [r for r in rows if r["ok"]]
    duration = max(r["ended_s"] for r in rows) - min(r["started_s"] for r in rows)
    for r in rows:
        r["conforming_standard"], r["conforming_strict"] = conforming(
            r, args.slo_ttft_ms / 1e3, args.slo_tpot_ms / 1e3, args.strict_max_itl_s)
    n_std = sum(r["conforming_standard"] for r in rows)
    n_strict = sum(r["conforming_strict"] for r in rows)
    in_toks = sum(r["prompt_tokens"] or 0 for r in good)
    out_toks = sum(r["output_tokens"] or 0 for r in good)
    e2es = [r["e2e_s"] for r in good]
    buckets = error_bucket_counts(rows)
    res = {**label, **admission_summary(rows),
           "achieved_qps": len(good) / duration, "request_throughput_per_s": len(good) / duration,
           "input_tokens_per_s": in_toks / duration, "output_tokens_per_s": out_toks / duration,
           "total_tokens_per_s": (in_toks + out_toks) / duration, "success_rate": len(good) / len(rows),
           "goodput_per_s": n_std / duration, "goodput_tokens_per_s": token_goodput(rows, duration),
           "slo_standard_rate": n_std / len(rows), "slo_standard_rate_ci95": list(wilson_ci(n_std, len(rows))),
           "slo_strict_rate": n_strict / len(rows), "slo_strict_rate_ci95": list(wilson_ci(n_strict, len(rows))),
           "counts": {"attempted": len(rows), "ok": len(good), "conforming_standard": n_std,
                      "conforming_strict": n_strict, **buckets},
           "error_buckets": buckets, "slo_ttft_ms": args.slo_ttft_ms, "slo_tpot_ms": args.slo_tpot_ms,
           "strict_max_itl_s": args.strict_max_itl_s, "max_concurrency": max_conc, "duration_s": duration,
           "e2e_cv": coefficient_of_variation(e2es), "p99_reference_only": len(rows) < 500,
           "mixed_steps": delta.get("engine_mixed_steps_total", 0.0),
           "prefill_steps": delta.get("engine_prefill_steps_total", 0.0),
           "decode_steps": delta.get("engine_decode_steps_total", 0.0),
           "preemptions": delta.get("scheduler_preemptions_total", 0.0)}
    res["slo_success_rate"] = res["slo_standard_rate"]
    ptoks = [r["prompt_tokens"] for r in good if r["prompt_tokens"] is not None]
    if ptoks:
        res.update({"prompt_tokens_min": min(ptoks), "prompt_tokens_p50": percentile(ptoks, 0.5, "linear"),
                    "prompt_tokens_max": max(ptoks)})
    hits, all_prompt = delta.get("kv_prefix_hit_tokens_total", 0.0), sum(r["prompt_tokens"] or 0 for r in rows)
    res["prefix_cache_hit_rate"] = hits / all_prompt if hits and all_prompt else 0.0
    if gpu_max:
        res["gpu_mem_mib_max"] = [g["mem_mib"] for g in gpu_max]
        res["gpu_util_pct_max"] = [g["util_pct"] for g in gpu_max]
    for name, vals in (("ttft", [r["ttft_s"] for r in good]), ("tpot", [r["tpot_s"] for r in good]),
                       ("itl", [g for r in good for g in r["itls_s"]]), ("e2e", e2es)):
        res.update(distribution(vals, name))
    outs = [r["output_tokens"] for r in good if r.get("output_tokens") is not None]
    res["output_tokens_p50"], res["output_tokens_p95"] = percentile(outs, 0.5), percentile(outs, 0.95)
    s2f = [r["server_ttft_s"] - r["server_queue_s"] for r in rows
           if r.get("server_ttft_s") is not None and r.get("server_queue_s") is not None]
    res.update(distribution(s2f, "scheduled_to_first_token"))
    queues = [r["server_queue_s"] for r in rows if r.get("server_queue_s") is not None]
    if queues:
        res.update({"queue_p50_s": percentile(queues, 0.5, "linear"), "queue_p95_s": percentile(queues, 0.95, "linear"),
                    "queue_samples": len(queues)})
    return res


def aggregate(summaries: list[dict], key_fields: tuple) -> list[dict]:
    """Pooled SLO rates (Wilson intervals) and per-repeat spread of each load point."""
    groups: dict[tuple, list] = {}
    for s in summaries:
        groups.setdefault(tuple(s[k] for k in key_fields), []).append(s)
    out = []
    for key, rows in sorted(groups.items(), key=lambda kv: str(kv[0])):
        att = sum(r["counts"]["attempted"] for r in rows)
        std = sum(r["counts"]["conforming_standard"] for r in rows)
        strict = sum(r["counts"]["conforming_strict"] for r in rows)
        e = {**dict(zip(key_fields, key)), "repeats": [r["repeat"] for r in rows],
             "slo_standard_rate_per_repeat": [r["slo_standard_rate"] for r in rows],
             "slo_strict_rate_per_repeat": [r["slo_strict_rate"] for r in rows],
             "slo_standard_rate_ci95": list(wilson_ci(std, att)), "slo_strict_rate_ci95": list(wilson_ci(strict, att)),
             "achieved_qps_median": percentile([r["achieved_qps"] for r in rows], 0.5, "linear")}
        counts = {f: sum(r["admission_counts"][f] for r in rows) for f in rows[0]["admission_counts"]}
        e.update({"admission_counts": counts, "reject_429_rate": counts["reject_429"] / att if att else None,
                  "admitted_slo_standard_rate": counts["conforming_standard"] / counts["admitted"]
                  if counts["admitted"] else None})
        out.append(e)
    return out


# ------------------------------------------------------------------ driver
async def async_main(args) -> dict:
    import httpx

    args.shape = RequestShape(args)  # its semaphore belongs to this event loop
    sampler = GpuSampler(args.gpu_sample_interval_s, enabled=not args.no_gpu_sample)
    sampler.start()
    tokenizer = None
    if args.tokenizer:
        from b200moe.utils.tokenizer import load_tokenizer
        tokenizer = load_tokenizer(args.tokenizer, vocab_size=1 << 20, eos_token_id=None)
    words = {"fixed": args.prompt_words}
    calibration = None
    if args.prompt_tokens:
        if tokenizer is None:
            raise SystemExit("--prompt-tokens needs --tokenizer")
        targets = {"fixed": args.prompt_tokens} if args.prompt_mode != "mixed" else \
            {"short": max(64, args.prompt_tokens // 4), "medium": args.prompt_tokens, "long": 2 * args.prompt_tokens}
        mode = "unique" if args.prompt_mode == "mixed" else args.prompt_mode
        calibration = {b: dict(zip(("prompt_words", "measured_tokens"),
                                   calibrate_words(tokenizer, args.prompt_word, mode, args.seed, t)), target_tokens=t)
                       for b, t in targets.items()}
        words = {b: c["prompt_words"] for b, c in calibration.items()}
    elif args.prompt_mode == "mixed":
        words = {"short": max(16, args.prompt_words // 4), "medium": args.prompt_words, "long": 2 * args.prompt_words}

    summaries, records = [], []
    limits = httpx.Limits(max_connections=None, max_keepalive_connections=None)
    try:
        async with httpx.AsyncClient(limits=limits, timeout=None) as client:
            for repeat in range(1, args.repeats + 1):
                seed = repeat_prompt_seed(args.seed, repeat, args.prompt_seed_per_repeat)

                def prompt_for(rid, seed=seed):
                    if args.prompt_dist == "lognormal":
                        return lognormal_prompt(seed, rid, args.prompt_median, args.prompt_sigma, args.prompt_min,
                                                args.prompt_max, args.prompt_vocab)
                    if args.prompt_mode == "mixed":
                        return build_prompt(args.prompt_word, words[mixed_bucket(abs(rid))], "unique", seed, rid)
                    return build_prompt(args.prompt_word, words["fixed"], args.prompt_mode, seed, rid)

                for pi, frac in enumerate(args.fractions):
                    label_phase = f"r{repeat}-p{pi}"
                    sampler.phase = label_phase
                    if args.mode == "poisson":
                        rows, b, a, mc = await run_point_poisson(client, args, frac, pi, repeat, prompt_for,
                                                                 tokenizer)
                        label = {"mode": "poisson", "load_fraction": frac, "target_qps": args.max_qps * frac,
                                 "repeat": repeat}
                    else:
                        rows, b, a, mc = await run_point_concurrency(client, args, frac, pi, repeat, prompt_for,
                                                                     tokenizer)
                        label = {"mode": "concurrency", "concurrency": int(frac), "repeat": repeat}
                    sampler.phase = "idle"
                    s = summarize(rows, mc, metrics_delta(b, a), args, label, sampler.max_for(label_phase))
                    s["metrics_before"], s["metrics_after"] = b, a
                    summaries.append(s)
                    records.extend(rows)
                    print(f"[online] {json.dumps({k: s[k] for k in ('repeat', 'achieved_qps', 'output_tokens_per_s', 'slo_standard_rate', 'ttft_p50_s', 'tpot_p50_s')})}",
                          flush=True)
    finally:
        sampler.stop()
    keys = ("mode", "load_fraction") if args.mode == "poisson" else ("mode", "concurrency")
    payload = {"schema_version": SCHEMA_VERSION, "args": {k: v for k, v in vars(args).items()},
               "prompt_calibration": calibration, "points": summaries, "aggregate": aggregate(summaries, keys),
               "records": records, "gpu_samples": sampler.samples}
    out = Path(args.output)
    out.parent.mkdir(parents=True, exist_ok=True)
    out.write_text(json.dumps(payload, indent=2, default=str))
    print(f"[online] wrote {out}")
    return payload


def parse_args(argv=None):
    p = argparse.ArgumentParser(description="online serving benchmark (HTTP streaming client)")
    p.add_argument("--base-url", default="http://127.0.0.1:8000")
    p.add_argument("--model", required=True)
    p.add_argument("--tokenizer", help="local tokenizer for prompt calibration / usage fallback")
    p.add_argument("--mode", choices=("poisson", "concurrency"), default="poisson")
    p.add_argument("--concurrency", type=lambda v: [int(x) for x in v.split(",")], default=None,
                   help="alias for --mode concurrency --fractions LIST (absolute levels)")
    p.add_argument("--max-qps", type=float, default=0.87)
    p.add_argument("--fractions", type=lambda v: [float(x) for x in v.split(",")], default=[0.25, 0.5, 0.75, 0.9])
    p.add_argument("--requests", type=int, default=128)
    p.add_argument("--warmup-requests", type=int, default=4)
    p.add_argument("--max-tokens", type=int, default=128)
    p.add_argument("--prompt-words", type=int, default=128)
    p.add_argument("--prompt-tokens", type=int, default=0)
    p.add_argument("--prompt-word", default="benchmark")
    p.add_argument("--prompt-mode", choices=("shared", "unique", "mixed"), default="shared")
    p.add_argument("--prompt-seed-per-repeat", action="store_true")
    p.add_argument("--arrival-pattern", choices=("fixed", "poisson"), default="poisson")
    p.add_argument("--seed", type=int, default=20261026)
    p.add_argument("--slo-ttft-ms", type=float, default=2000.0)
    p.add_argument("--slo-tpot-ms", type=float, default=500.0)
    p.add_argument("--strict-max-itl-s", type=float, default=1.0)
    p.add_argument("--repeats", type=int, default=1)
    p.add_argument("--request-timeout-s", type=float, default=120.0)
    p.add_argument("--duration", type=float, default=None)
    p.add_argument("--gpu-sample-interval-s", type=float, default=2.0)
    p.add_argument("--no-gpu-sample", action="store_true")
    p.add_argument("--output", default="online_benchmark.json")
    p.add_argument("--workload", choices=sorted(WORKLOADS), default=None,
                   help="preset prompt / output / sampling / concurrency of a named workload")
    p.add_argument("--prompt-dist", choices=("words", "lognormal"), default="words")
    p.add_argument("--prompt-median", type=float, default=1500.0)
    p.add_argument("--prompt-sigma", type=float, default=0.6)
    p.add_argument("--prompt-min", type=int, default=128)
    p.add_argument("--prompt-max", type=int, default=8192)
    p.add_argument("--prompt-vocab", type=int, default=32000, help="token ids are drawn below this")
    p.add_argument("--output-len-range", type=lambda v: tuple(int(x) for x in v.split(",")), default=None,
                   help="LO,HI: per-request max_tokens uniform in [LO, HI], with ignore_eos")
    p.add_argument("--temperature", type=float, default=0.0)
    p.add_argument("--top-p", type=float, default=1.0)
    p.add_argument("--max-concurrency", type=int, default=0, help="cap on in-flight Poisson requests (0: none)")
    pre, _ = p.parse_known_args(argv)
    if pre.workload:
        p.set_defaults(**WORKLOADS[pre.workload])
    args = p.parse_args(argv)
    if args.output_len_range is not None and (len(args.output_len_range) != 2
                                              or not 0 < args.output_len_range[0] <= args.output_len_range[1]):
        p.error("--output-len-range takes LO,HI with 0 < LO <= HI")
    if not 0 < args.prompt_min <= args.prompt_max:
        p.error("--prompt-min / --prompt-max must satisfy 0 < min <= max")
    if not (args.max_qps > 0 and args.requests > 0 and args.warmup_requests >= 0 and args.repeats >= 1):
        p.error("max-qps, requests, repeats must be positive; warmup-requests >= 0")
    if not all(f > 0 for f in args.fractions):
        p.error("fractions must be positive")
    if args.concurrency is not None:
        args.mode, args.fractions = "concurrency", [float(c) for c in args.concurrency]
    return args


def main(argv=None):
    return asyncio.run(async_main(parse_args(argv)))


if __name__ == "__main__":
    main()
