"""Offline benchmark driver: a correctness gate, then a throughput / latency sweep.

    python -m b200moe.bench_offline --model qwen3-30b-a3b --random-init \
        --batches 1,8,64,256 --prompt-len 1024 --output-len 256 --output sweep.json

Behaviour follows the reference's offline driver (scripts/p2_benchmark.py:34-448):

* **Gate before perf.** Four fixed prompts are decoded greedily
  (``--verify-max-tokens``) on every ``--verify-backends`` MoE backend: one
  discarded warm-up, then ``--verify-repeats`` runs with the prefix cache
  cleared between them (new block layout).  Hard failures: a backend that is
  not deterministic across repeats, or (with ``--reference-outputs``) that
  differs from the frozen reference.  Agreement between backends is reported;
  it is a hard gate only with ``--strict-cross-backend``, because the
  per-expert ``loop`` accumulates in a different order from the grouped
  kernel and may flip near-tied tokens.  ``--freeze-reference PATH`` writes
  the gate's outputs as a new frozen reference.
* **Matrix.** attention backend x cache mode x MoE backend x batch, each point
  one untimed pass plus ``--repeats`` timed passes through ``LLM.generate``.
  Cache modes: ``none``; ``cold`` (prefix cache cleared before each repeat);
  ``hot`` (kept).  Prompts share ``--shared-prefix-len`` tokens.
* **Probe phase** (``--probe-batches``): the same in one model load with a
  long shared prefix, to measure prefix-cache hits.
* ``--workload offline|longctx|235b`` presets the headline family's shapes
  (256 x 1024 -> 256 on Qwen3-30B-A3B; 8 x 32768 -> 512 with 256-token
  blocks, with ``--kv-cache-dtype int8`` and ``--kv-offload`` variants;
  Qwen3-235B-A22B 128 x 2048 -> 256); explicit flags override the preset.
* Every record streams to a JSONL file as it completes; the JSON payload
  (schema 2: records, per-point summary with median / CV, verification,
  provenance, environment) is written at the end.

Each record also carries the engine's device time for the pass (CUDA events
around every step, max over ranks), which the reference does not measure.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import platform
import random
import statistics
import subprocess
import time
from pathlib import Path

from b200moe.benchmarking import coefficient_of_variation, percentile

VERIFY_PROMPTS = [
    "introduce yourself",
    "list all prime numbers within 100",
    "请用三句话解释什么是 Mixture of Experts。",
    "请用 Python 写一个快速排序，附注释。",
]
CACHE_MODES = ("none", "cold", "hot")
# named workloads of the headline benchmark family; explicit flags override them
WORKLOADS = {
    # 8 concurrent 32k-token prompts, 512 decode tokens, 256-token KV blocks (bf16 or
    # --kv-cache-dtype int8; --kv-offload with --num-kvcache-blocks below the demand
    # exercises host offload once HBM blocks run out)
    "longctx": dict(model="qwen3-30b-a3b", batches="8", prompt_len=32768, output_len=512, kvcache_block_size=256,
                    max_num_batched_tokens=32768),
    # Qwen3-235B-A22B: 128 concurrent 2048-token prompts, 256 output tokens
    "235b": dict(model="qwen3-235b-a22b", batches="128", prompt_len=2048, output_len=256, kvcache_block_size=256),
    # the offline headline: 256 x 1024 -> 256 on Qwen3-30B-A3B
    "offline": dict(model="qwen3-30b-a3b", batches="256", prompt_len=1024, output_len=256, kvcache_block_size=256),
}


def make_prompts(batch: int, prompt_len: int, vocab_size: int, seed: int, shared_prefix_len: int = 0):
    rng = random.Random(seed)
    shared = [rng.randrange(vocab_size) for _ in range(shared_prefix_len)]
    return [shared + [rng.randrange(vocab_size) for _ in range(prompt_len - shared_prefix_len)]
            for _ in range(batch)]


def numeric_delta(before: dict, after: dict) -> dict:
    return {k: v - before.get(k, 0) for k, v in after.items()
            if isinstance(v, (int, float)) and isinstance(before.get(k, 0), (int, float))}


def file_sha256(path) -> str | None:
    p = Path(path)
    return hashlib.sha256(p.read_bytes()).hexdigest() if p.is_file() else None


def git_commit() -> str | None:
    try:
        return subprocess.check_output(["git", "rev-parse", "HEAD"], cwd=Path(__file__).resolve().parents[1],
                                       text=True, stderr=subprocess.DEVNULL).strip()
    except (OSError, subprocess.CalledProcessError):
        return None


def _csv(s: str) -> list[str]:
    return [x.strip() for x in s.split(",") if x.strip()]


def run_verification(llm, sp_cls, backends, max_tokens, repeats, reference_path=None, strict_cross=False):
    """Determinism / frozen-reference / cross-backend gate; raises SystemExit on a hard failure."""
    reference = None
    if reference_path:
        reference = [list(r["token_ids"]) for r in json.loads(Path(reference_path).read_text())]
    params = sp_cls(temperature=0.0, max_tokens=max_tokens, ignore_eos=True)
    result = {"prompts": VERIFY_PROMPTS, "reference": reference_path, "repeats": repeats, "backends": {}}
    failures = []
    for backend in backends:
        llm.executor.call("set_moe_backend", backend)
        warm = [list(o["token_ids"]) for o in llm.generate(VERIFY_PROMPTS, params, use_tqdm=False)]
        runs = []
        for r in range(repeats):
            if r:
                llm.scheduler.clear_prefix_cache()
            runs.append([list(o["token_ids"]) for o in llm.generate(VERIFY_PROMPTS, params, use_tqdm=False)])
        entry = {"warmup": warm, "runs": runs, "deterministic": all(x == runs[0] for x in runs),
                 "warmup_matches_steady": warm == runs[0]}
        if not entry["deterministic"]:
            failures.append(f"{backend}: repeat nondeterminism")
        if reference is not None:
            entry["reference_matches"] = [x == reference for x in runs]
            if not all(entry["reference_matches"]):
                failures.append(f"{backend}: frozen reference mismatch")
        result["backends"][backend] = entry
        print(f"[verify] {backend} deterministic={entry['deterministic']} "
              f"reference_matches={entry.get('reference_matches')}", flush=True)
    base = backends[0]
    for b in backends[1:]:
        agree = [x == y for x, y in zip(result["backends"][base]["runs"][0], result["backends"][b]["runs"][0])]
        result["backends"][b]["matches_" + base] = agree
        print(f"[verify] {b} vs {base} prompt matches={agree}", flush=True)
        if strict_cross and not all(agree):
            failures.append(f"{b}: differs from {base}")
    llm.executor.call("set_moe_backend", backends[0])
    result["deterministic_all"] = all(e["deterministic"] for e in result["backends"].values())
    result["passed"] = not failures
    result["failures"] = failures
    if failures:
        raise SystemExit("[verify] hard gate failed: " + "; ".join(failures))
    return result


def parse_args(argv=None):
    p = argparse.ArgumentParser(description="offline benchmark sweep with a correctness gate")
    p.add_argument("--model", default="qwen3-30b-a3b")
    p.add_argument("--random-init", action="store_true", help="random weights of the named architecture")
    p.add_argument("--tensor-parallel-size", type=int, default=1)
    p.add_argument("--batches", default="1,2,4,8,16,32,64")
    p.add_argument("--prompt-len", type=int, default=128)
    p.add_argument("--output-len", type=int, default=128)
    p.add_argument("--repeats", type=int, default=3)
    p.add_argument("--moe-backends", default="fused")
    p.add_argument("--attention-backends", default="paged")
    p.add_argument("--graph-modes", default="", help="comma list of eager|graphs (decode CUDA graphs A/B)")
    p.add_argument("--expert-placement", choices=("linear", "round_robin", "profiled"), default="linear")
    p.add_argument("--expert-map-path")
    p.add_argument("--scheduler-policy", choices=("fcfs", "stall_free", "stall_free_lpm", "lpm"), default="fcfs")
    p.add_argument("--enforce-eager", action="store_true")
    p.add_argument("--kvcache-block-size", type=int, default=256)
    p.add_argument("--max-num-batched-tokens", type=int, default=16384)
    p.add_argument("--output", default="offline_benchmark.json")
    p.add_argument("--jsonl")
    p.add_argument("--shared-prefix-len", type=int, default=0)
    p.add_argument("--cache-modes", "--cache-mode", dest="cache_modes", default="none")
    p.add_argument("--skip-verification", action="store_true")
    p.add_argument("--reference-outputs", default=None, help="frozen reference JSON for the gate")
    p.add_argument("--freeze-reference", default=None, help="write the gate's outputs here as a new reference")
    p.add_argument("--verify-max-tokens", type=int, default=8)
    p.add_argument("--verify-repeats", type=int, default=3)
    p.add_argument("--verify-backends", default="fused")
    p.add_argument("--strict-cross-backend", action="store_true")
    p.add_argument("--probe-batches", default="")
    p.add_argument("--probe-prompt-len", type=int, default=512)
    p.add_argument("--probe-shared-prefix-len", type=int, default=384)
    p.add_argument("--probe-cache-modes", default="cold,hot")
    p.add_argument("--device", default=None)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--workload", choices=sorted(WORKLOADS), default=None,
                   help="preset model / batch / lengths of a named workload")
    p.add_argument("--kv-cache-dtype", choices=("bf16", "int8"), default="bf16")
    p.add_argument("--kv-int8-mode", choices=("token", "channel"), default="token")
    p.add_argument("--kv-offload", action="store_true", help="host KV offload of evicted prefix blocks")
    p.add_argument("--kv-offload-host-blocks", type=int, default=256)
    p.add_argument("--num-kvcache-blocks", type=int, default=-1, help="-1: size the pool from free memory")
    p.add_argument("--attention-parallel", choices=("dp", "tp"), default="dp")
    p.add_argument("--prefill-chunk-size", type=int, default=0)
    pre, _ = p.parse_known_args(argv)
    if pre.workload:
        p.set_defaults(**WORKLOADS[pre.workload])
    args = p.parse_args(argv)
    args.cache_modes = _csv(args.cache_modes)
    args.probe_cache_modes = _csv(args.probe_cache_modes)
    for m in args.cache_modes + args.probe_cache_modes:
        if m not in CACHE_MODES:
            p.error(f"cache mode must be one of {CACHE_MODES}")
    if not 0 <= args.shared_prefix_len <= args.prompt_len:
        p.error("--shared-prefix-len must lie in [0, prompt-len]")
    if any(m != "none" for m in args.cache_modes) and args.shared_prefix_len == 0:
        p.error("cache modes cold/hot need --shared-prefix-len")
    if _csv(args.probe_batches) and any(m != "none" for m in args.probe_cache_modes) \
            and args.probe_shared_prefix_len < args.kvcache_block_size:
        p.error("the prefix-cache probe needs a shared prefix of at least one KV block")
    return args


def engine_kwargs(args) -> dict:
    """``LLM(**kw)`` for the parsed options."""
    batches = [int(x) for x in _csv(args.batches)]
    probe_batches = [int(x) for x in _csv(args.probe_batches)]
    max_len = max(args.prompt_len, args.probe_prompt_len if probe_batches else 0) + args.output_len + 16
    kw = dict(tensor_parallel_size=args.tensor_parallel_size, enforce_eager=args.enforce_eager,
              moe_backend=_csv(args.moe_backends)[0], attention_backend=_csv(args.attention_backends)[0],
              expert_placement=args.expert_placement, expert_map_path=args.expert_map_path,
              scheduler_policy=args.scheduler_policy, max_model_len=max(max_len, 256),
              max_num_seqs=max(batches + probe_batches + [len(VERIFY_PROMPTS)]),
              max_num_batched_tokens=args.max_num_batched_tokens, kvcache_block_size=args.kvcache_block_size,
              seed=args.seed, kv_cache_dtype=args.kv_cache_dtype, kv_int8_mode=args.kv_int8_mode,
              attention_parallel=args.attention_parallel)
    if args.kv_offload:
        kw.update(kv_offload_enabled=True, kv_offload_host_blocks=args.kv_offload_host_blocks)
    if args.num_kvcache_blocks > 0:
        kw["num_kvcache_blocks"] = args.num_kvcache_blocks
    if args.prefill_chunk_size > 0:
        kw["prefill_chunk_size"] = args.prefill_chunk_size
    if args.random_init:
        kw["random_init"] = "seeded"
    if args.device:
        kw["device"] = args.device
    return kw


def main(argv=None):
    args = parse_args(argv)
    from b200moe import LLM, SamplingParams

    batches = [int(x) for x in _csv(args.batches)]
    probe_batches = [int(x) for x in _csv(args.probe_batches)]
    backends = _csv(args.moe_backends)
    attn_backends = _csv(args.attention_backends)
    graph_modes = _csv(args.graph_modes) or [None]
    if any(g not in (None, "eager", "graphs") for g in graph_modes):
        raise SystemExit("--graph-modes takes eager and/or graphs")
    graph_mem: dict[str, int] = {}
    kw = engine_kwargs(args)
    llm = LLM(args.model, **kw)
    vocab = llm.config.hf_config.vocab_size
    params = SamplingParams(temperature=0.0, max_tokens=args.output_len, ignore_eos=True)
    records, verification = [], None
    jsonl_path = Path(args.jsonl) if args.jsonl else Path(args.output).with_suffix(".jsonl")
    jsonl_path.parent.mkdir(parents=True, exist_ok=True)
    fh = jsonl_path.open("w", encoding="utf-8")
    try:
        if not args.skip_verification:
            ref = args.reference_outputs
            if ref and not Path(ref).is_file():
                raise SystemExit(f"[verify] frozen reference missing: {ref}")
            verification = run_verification(llm, SamplingParams, _csv(args.verify_backends),
                                            args.verify_max_tokens, args.verify_repeats, ref,
                                            args.strict_cross_backend)
            if args.freeze_reference:
                runs = verification["backends"][_csv(args.verify_backends)[0]]["runs"][0]
                Path(args.freeze_reference).write_text(json.dumps(
                    [{"prompt": p, "token_ids": t} for p, t in zip(VERIFY_PROMPTS, runs)], indent=1))

        def measure(attn, backend, batch, prompt_len, shared, cache_mode, phase, graph_mode=None):
            llm.executor.call("set_attention_backend", attn)
            llm.executor.call("set_moe_backend", backend)
            if graph_mode is not None:
                llm.executor.call("set_cuda_graphs", graph_mode == "graphs")
                graph_mem[graph_mode] = max(llm.executor.call_all("memory_reserved"))
            else:
                graph_mode = "eager" if args.enforce_eager else "graphs"
            prompts = make_prompts(batch, prompt_len, vocab, seed=batch, shared_prefix_len=shared)
            llm.generate(prompts, params, use_tqdm=False)
            for rep in range(args.repeats):
                if cache_mode in ("cold", "none"):
                    # "none": no measured pass may reuse the warm-up's (or another pass's) prompt KV
                    llm.scheduler.clear_prefix_cache()
                before = llm.scheduler.metrics()
                llm.executor.call_all("reset_step_timing")
                t0 = time.perf_counter()
                outs = llm.generate(prompts, params, use_tqdm=False)
                elapsed = time.perf_counter() - t0
                device_s = max(llm.executor.call_all("step_device_ms")) / 1e3
                after = llm.scheduler.metrics()
                ttfts = [o["metrics"]["ttft_s"] for o in outs]
                tpots = [o["metrics"]["tpot_s"] for o in outs]
                itls = [g for o in outs for g in o["metrics"]["itls_s"]]
                out_toks = sum(len(o["token_ids"]) for o in outs)
                in_toks = sum(o["metrics"]["prompt_tokens"] for o in outs)
                rec = {"phase": phase, "attention_backend": attn, "backend": backend, "graph_mode": graph_mode,
                       "batch": batch,
                       "repeat": rep, "prompt_len": prompt_len, "output_len": args.output_len,
                       "shared_prefix_len": shared, "cache_mode": cache_mode, "cache_metrics_before": before,
                       "cache_metrics_after": after, "cache_metrics_delta": numeric_delta(before, after),
                       "elapsed_s": elapsed, "device_s": device_s, "input_tokens": in_toks,
                       "output_tokens": out_toks, "input_tokens_per_s": in_toks / elapsed,
                       "output_tokens_per_s": out_toks / elapsed,
                       "total_tokens_per_s": (in_toks + out_toks) / elapsed,
                       "device_output_tokens_per_s": out_toks / device_s if device_s > 0 else None,
                       "ttft_p50_s": percentile(ttfts, 0.5), "ttft_p95_s": percentile(ttfts, 0.95),
                       "tpot_p50_s": percentile(tpots, 0.5), "tpot_p95_s": percentile(tpots, 0.95),
                       "itl_p50_s": percentile(itls, 0.5), "itl_p95_s": percentile(itls, 0.95),
                       "requests": [{**o["metrics"], "token_ids": o["token_ids"]} for o in outs]}
                records.append(rec)
                fh.write(json.dumps(rec, sort_keys=True) + "\n")
                fh.flush()
                print("[bench]", json.dumps({k: v for k, v in rec.items() if k != "requests"}, sort_keys=True),
                      flush=True)

        for attn in attn_backends:
            for cm in args.cache_modes:
                for be in backends:
                    for gm in graph_modes:
                        for b in batches:
                            measure(attn, be, b, args.prompt_len, args.shared_prefix_len, cm, "matrix", gm)
        for attn in attn_backends:
            for be in backends:
                for b in probe_batches:
                    for cm in args.probe_cache_modes:
                        measure(attn, be, b, args.probe_prompt_len, args.probe_shared_prefix_len, cm, "probe")
    finally:
        fh.close()
        llm.exit()

    summary = []
    keys = ("phase", "attention_backend", "cache_mode", "backend", "graph_mode", "batch")
    groups: dict[tuple, list] = {}
    for r in records:
        groups.setdefault(tuple(r[k] for k in keys), []).append(r)
    for key, rows in groups.items():
        thr = [r["output_tokens_per_s"] for r in rows]
        med = lambda f: statistics.median(r[f] for r in rows if r[f] is not None) \
            if any(r[f] is not None for r in rows) else None
        summary.append({**dict(zip(keys, key)), "prompt_len": rows[0]["prompt_len"],
                        "shared_prefix_len": rows[0]["shared_prefix_len"],
                        "throughput_median": statistics.median(thr), "throughput_cv": coefficient_of_variation(thr),
                        "device_throughput_median": med("device_output_tokens_per_s"),
                        "ttft_p95_median_s": med("ttft_p95_s"), "tpot_p95_median_s": med("tpot_p95_s"),
                        "itl_p95_median_s": med("itl_p95_s")})
    model_dir = Path(args.model)
    payload = {
        "schema_version": 2, "model": args.model, "random_init": args.random_init, "moe_backends": backends,
        "attention_backends": attn_backends, "expert_placement": args.expert_placement,
        "scheduler_policy": args.scheduler_policy, "shared_prefix_len": args.shared_prefix_len,
        "cache_modes": args.cache_modes, "verification": verification,
        "provenance": {"git_commit": git_commit(),
                       "model_config_sha256": file_sha256(model_dir / "config.json"),
                       "tokenizer_config_sha256": file_sha256(model_dir / "tokenizer_config.json"),
                       "reference_sha256": file_sha256(args.reference_outputs) if args.reference_outputs else None},
        "environment": {"python": platform.python_version(), "platform": platform.platform(),
                        "cuda_visible_devices": os.environ.get("CUDA_VISIBLE_DEVICES")},
        "records": records, "summary": summary,
        "graph_memory_delta_gib": (graph_mem["graphs"] - graph_mem["eager"]) / 2 ** 30
        if {"graphs", "eager"} <= graph_mem.keys() else None,
    }
    Path(args.output).write_text(json.dumps(payload, indent=2), encoding="utf-8")
    print(f"[bench] wrote {args.output} and {jsonl_path}")
    return payload


if __name__ == "__main__":
    main()
