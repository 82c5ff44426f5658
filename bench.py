"""Headline benchmark: offline output tok/s of Qwen3-30B-A3B-FP8.

Workload: 256 requests with 1024-token uniform-random
prompts, 256 greedy output tokens each; random-init e4m3 weights with
128x128 block scales (no checkpoint download), bf16 activations.  One bench
"step" is one full pass of the workload through ``LLM.generate``.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200moe|reference]

Reported:
  value          output tokens / device time of the K timed passes.  Device
                 time = sum over engine steps of the CUDA-event time between
                 the start of the step's input upload and the end of its
                 sampling, max over ranks (host-side scheduling excluded).
  e2e.value      the same tokens over the host wall clock of the K calls to
                 ``LLM.generate`` (public API: pinned H2D of every step's
                 packed inputs, D2H of the sampled ids, scheduling).
  gpu_launches   native kernels launched in the timed region (counted by the
                 extension wrappers; graph replays count their captured kernels).
Weights (30 GB) dwarf the 126 MB L2, so no explicit L2 flush is done.
For N > 1 (torchrun) rank 0 drives the engine and ranks 1..N-1 serve as its
expert-parallel workers.
"""
from __future__ import annotations

import argparse
import json
import os
import random
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
BASELINE_TOKS = None  # the reference publishes no number for this config on this hardware


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=int(os.environ.get("WORLD_SIZE", "1")))
    p.add_argument("--steps", type=int, default=2)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["b200moe", "reference"], default="b200moe")
    p.add_argument("--model", default="qwen3-30b-a3b")
    p.add_argument("--num-requests", type=int, default=256)
    p.add_argument("--input-len", type=int, default=1024)
    p.add_argument("--output-len", type=int, default=256)
    p.add_argument("--max-num-batched-tokens", type=int, default=16384)
    p.add_argument("--scheduler-policy", default="fcfs")
    p.add_argument("--attention-parallel", default="dp")
    p.add_argument("--enforce-eager", action="store_true")
    p.add_argument("--scheduler-overlap", type=int, choices=(0, 1), default=1,
                   help="schedule step N+1 on the host while step N runs on the GPU")
    p.add_argument("--seed", type=int, default=0)
    return p.parse_args()


def workload(args, pass_index: int = 0):
    """Uniform-random prompts; every pass (warm-up or timed) draws its own, so no
    pass reuses another's prompt KV through the prefix cache."""
    rng = random.Random(args.seed * 1_000_003 + pass_index)
    vocab = 151936
    return [[rng.randrange(vocab) for _ in range(args.input_len)] for _ in range(args.num_requests)]


METRIC = "output tok/s (Qwen3-30B-A3B FP8, EP8, 256 concurrent) + p50 TTFT/TPOT"


def reference_arm(args):
    sys.path.insert(0, os.path.join(ROOT, "baseline"))
    import reference_arm as ref
    return ref.run(args, lambda i: workload(args, i), METRIC)


def _parallelism(n: int, rep: dict) -> str:
    """Layout label from what the engine reports: data-parallel attention with the experts
    split by expert parallelism (``ep{n}+dp{n}-attn``), or head-sharded attention with the
    experts split and every partial summed across ranks (``tp{n}``)."""
    if rep.get("attention_parallel") == "tp":
        return f"tp{n}" + ("-fused-peer-sums" if rep.get("tp_fused") else "-nccl")
    return f"ep{n}+dp{n}-attn"


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    if args.gpus > 1 and rank != 0:
        # torchrun-launched non-driver ranks.  Both arms' engines run on rank 0 and
        # spawn their own process per GPU, so these ranks have nothing to do: they
        # exit at once, touching neither CUDA nor any store.  torchrun's agent ends
        # the job when every local rank has exited, and counts a clean early exit
        # as success, so nothing waits on a rendezvous that may never come.
        return 0
    if args.impl == "reference":
        return reference_arm(args)
    os.environ.setdefault("B200MOE_EP_STRICT", "1")  # the fused EP path runs, or the bench fails
    import torch
    from b200moe import LLM, SamplingParams, ops
    from b200moe.utils.gpu_clock import ClockSampler

    sp = SamplingParams(temperature=0.0, max_tokens=args.output_len, ignore_eos=True)
    t_init = time.perf_counter()
    llm = LLM(args.model, tensor_parallel_size=args.gpus, max_num_seqs=max(args.num_requests, 1),
              max_num_batched_tokens=args.max_num_batched_tokens, max_model_len=args.input_len + args.output_len + 16,
              kvcache_block_size=256, scheduler_policy=args.scheduler_policy,
              attention_parallel=args.attention_parallel, enforce_eager=args.enforce_eager, seed=args.seed,
              scheduler_overlap=bool(args.scheduler_overlap), random_init="seeded")
    init_s = time.perf_counter() - t_init
    runners = llm.executor
    for i in range(args.warmup):
        llm.generate(workload(args, i), sp, use_tqdm=False)
    timed_prompts = [workload(args, args.warmup + i) for i in range(args.steps)]  # built before the clock starts
    torch.cuda.synchronize()
    ops.reset_launch_count()
    runners.call("reset_step_timing")
    h2d0 = runners.runner.h2d_bytes
    steps0 = llm.step_count
    with ClockSampler(list(range(args.gpus))) as clk:
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        total_out = 0
        for prompts in timed_prompts:
            outs = llm.generate(prompts, sp, use_tqdm=False)
            total_out += sum(len(o["token_ids"]) for o in outs)
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
    dev_ms = max(runners.call_all("step_device_ms"))
    split = runners.call("step_device_split")  # rank 0: where the device time goes
    launches = sum(runners.call_all("launch_count"))
    par = runners.call_all("parallel_report")
    # the engine's actual layout, from rank 0's own report
    nsteps = llm.step_count - steps0
    h2d = (runners.runner.h2d_bytes - h2d0) / max(nsteps, 1)
    d2h = 4 * total_out / max(nsteps, 1)
    value = total_out / (dev_ms / 1e3)
    e2e = total_out / wall
    line = {
        "metric": METRIC,
        "value": round(value, 1), "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(dev_ms / args.steps, 2), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None if BASELINE_TOKS is None else round(value / BASELINE_TOKS, 3),
        "dtype": "bf16 activations, e4m3 block-scaled weights",
        "data": "synthetic uniform-random token ids; random-init weights (seeded)",
        "config": {"model": args.model, "global_batch": args.num_requests, "seq_len": args.input_len,
                   "output_len": args.output_len, "parallelism": _parallelism(args.gpus, par[0]),
                   "l2": "inputs larger than L2 (30 GB of weights per pass), no flush",
                   "prompts": "fresh uniform-random prompts every pass (no cross-pass prefix-cache hits)",
                   "scheduler_overlap": bool(args.scheduler_overlap),
                   "engine_steps_per_pass": nsteps // max(args.steps, 1), "init_s": round(init_s, 1),
                   "device_ms_split_rank0": {k: round(v, 1) if isinstance(v, float) else v for k, v in split.items()},
                   "ep_backend": par[0]["ep_backend"], "decode_graph_buckets": len(par[0]["decode_graphs"]),
                   "cuda_graphs": bool(par[0]["decode_graphs"])},
        "e2e": {"value": round(e2e, 1), "unit": "tok/s", "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h), "wall_s_per_pass": round(wall / args.steps, 3)},
        "gpu_launches": int(launches),
        "clocks": clk.summary(),
    }
    if any("ep_wait" in p for p in par):
        # device ms each rank's EP kernels waited, summed over the timed passes: per rank, the
        # total, and which peer it waited on longest (the straggler)
        line["ep_wait_ms"] = [
            {"rank": r, "dispatch": round(sum(p["ep_wait"]["dispatch_ms"]), 1),
             "combine": round(sum(p["ep_wait"]["combine_ms"]), 1),
             "worst_peer": max(range(len(p["ep_wait"]["dispatch_ms"])),
                               key=lambda q: p["ep_wait"]["dispatch_ms"][q] + p["ep_wait"]["combine_ms"][q])}
            for r, p in enumerate(par) if "ep_wait" in p]
    ttft = sorted(o["metrics"]["ttft_s"] for o in outs if o["metrics"]["ttft_s"] is not None)
    tpot = sorted(o["metrics"]["tpot_s"] for o in outs if o["metrics"]["tpot_s"] is not None)
    if ttft:
        line["p50_ttft_s"] = round(ttft[len(ttft) // 2], 4)
    if tpot:
        line["p50_tpot_s"] = round(tpot[len(tpot) // 2], 5)
    print(json.dumps(line), flush=True)
    llm.exit()
    return 0


if __name__ == "__main__":
    sys.exit(main())
