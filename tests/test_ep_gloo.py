"""Expert-parallel plumbing on CPU: two gloo ranks (spawned by the engine),
data-parallel attention, experts split across ranks; tokens must match the
single-rank engine (fp32 tiny model)."""
import random

import numpy as np
import pytest

from b200moe import LLM, SamplingParams


def _prompts(n=8, seed=0):
    rng = random.Random(seed)
    return [[rng.randrange(1024) for _ in range(rng.randint(16, 64))] for _ in range(n)]


def test_gloo_world2_matches_single_rank():
    kw = dict(device="cpu", kvcache_block_size=16, num_kvcache_blocks=128, max_num_batched_tokens=512,
              max_num_seqs=16, max_model_len=256, enforce_eager=True)
    sp = SamplingParams(temperature=0.0, max_tokens=16, ignore_eos=True)
    prompts = _prompts()
    one = LLM("tiny-moe", **kw)
    a = [o["token_ids"] for o in one.generate(prompts, sp, use_tqdm=False)]
    one.exit()
    two = LLM("tiny-moe", tensor_parallel_size=2, **kw)
    b = [o["token_ids"] for o in two.generate(prompts, sp, use_tqdm=False)]
    m = two.metrics()
    two.exit()
    assert m["kv_blocks_capacity"] == 2 * 128
    agree = np.mean([x == y for ra, rb in zip(a, b) for x, y in zip(ra, rb)])
    assert agree > 0.98, agree


def test_gloo_tensor_parallel_attention_matches_single_rank():
    """attention_parallel="tp": heads split over 2 gloo ranks, O-projection and
    expert partial sums all-reduced; tokens must match one rank."""
    kw = dict(device="cpu", kvcache_block_size=16, num_kvcache_blocks=128, max_num_batched_tokens=512,
              max_num_seqs=16, max_model_len=256, enforce_eager=True)
    sp = SamplingParams(temperature=0.0, max_tokens=16, ignore_eos=True)
    prompts = _prompts(seed=1)
    one = LLM("tiny-moe", random_init="seeded", **kw)
    a = [o["token_ids"] for o in one.generate(prompts, sp, use_tqdm=False)]
    one.exit()
    two = LLM("tiny-moe", tensor_parallel_size=2, attention_parallel="tp", random_init="seeded", **kw)
    heads = two.executor.call_all("kv_heads")
    b = [o["token_ids"] for o in two.generate(prompts, sp, use_tqdm=False)]
    two.exit()
    assert heads == [1, 1]  # tiny-moe has 2 KV heads: one per rank
    agree = np.mean([x == y for ra, rb in zip(a, b) for x, y in zip(ra, rb)])
    assert agree > 0.98, agree


def test_gloo_world2_launch_ahead_decode():
    """Two gloo ranks with the overlap pipeline: launch-ahead decode steps (each
    rank reads its own previous step's tokens on the device) match one rank."""
    kw = dict(device="cpu", kvcache_block_size=16, num_kvcache_blocks=128, max_num_batched_tokens=512,
              max_num_seqs=16, max_model_len=256, enforce_eager=True, random_init="seeded")
    rng = random.Random(2)
    prompts = _prompts(seed=2)
    sps = [SamplingParams(temperature=0.0, max_tokens=rng.randrange(4, 20), ignore_eos=True) for _ in prompts]
    one = LLM("tiny-moe", scheduler_overlap=False, **kw)
    a = [o["token_ids"] for o in one.generate(prompts, sps, use_tqdm=False)]
    one.exit()
    two = LLM("tiny-moe", tensor_parallel_size=2, scheduler_overlap=True, **kw)
    b = [o["token_ids"] for o in two.generate(prompts, sps, use_tqdm=False)]
    m = two.metrics()
    two.exit()
    assert m["engine_decode_feed_steps_total"] > 0
    assert [len(x) for x in a] == [len(x) for x in b]
    agree = np.mean([x == y for ra, rb in zip(a, b) for x, y in zip(ra, rb)])
    assert agree > 0.98, agree


def _offload_run(llm):
    rng = random.Random(9)
    shared = [rng.randrange(500) for _ in range(64)]
    group_a = [shared + [rng.randrange(500) for _ in range(16)] for _ in range(4)]
    group_b = [[rng.randrange(500) for _ in range(96)] for _ in range(12)]
    sp = SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True)
    try:
        first = [o["token_ids"] for o in llm.generate(group_a, sp, use_tqdm=False)]
        llm.generate(group_b, sp, use_tqdm=False)  # evicts group A's prefix to the host pool
        again = [o["token_ids"] for o in llm.generate(group_a, sp, use_tqdm=False)]
        return first, again, llm.metrics()
    finally:
        llm.exit()


@pytest.mark.parametrize("attention_parallel", ["dp", "tp"])
def test_gloo_world2_overlap_with_kv_offload(attention_parallel):
    """Two gloo ranks, overlap pipeline, a device pool small enough that the
    speculative schedule moves blocks to and from the host pool while a step
    is in flight: the workers' offload replies and step replies are matched
    by kind, and the tokens match one rank without offload."""
    kw = dict(device="cpu", kvcache_block_size=16, max_num_batched_tokens=256, max_num_seqs=8, max_model_len=256,
              enforce_eager=True, rank_timeout_s=60)
    ref, _, _ = _offload_run(LLM("tiny-moe", num_kvcache_blocks=64, **kw))
    first, again, m = _offload_run(LLM("tiny-moe", num_kvcache_blocks=24, kv_offload_enabled=True,
                                       kv_offload_host_blocks=64, tensor_parallel_size=2, scheduler_overlap=True,
                                       attention_parallel=attention_parallel, **kw))
    assert m["kv_offload_puts_total"] > 0 and m["kv_offload_revives_total"] > 0, m
    for got in (first, again):
        agree = np.mean([x == y for ra, rb in zip(ref, got) for x, y in zip(ra, rb)])
        assert agree > 0.98, agree


def test_gloo_world2_profile_snapshot_and_init_trace(monkeypatch, capfd):
    """Device-timed ranges switched on at run time on both ranks, gathered by
    the engine with the slowest rank per range; init milestones are timed on
    every rank and printed under B200MOE_TRACE_INIT."""
    monkeypatch.setenv("B200MOE_TRACE_INIT", "1")
    kw = dict(device="cpu", kvcache_block_size=16, num_kvcache_blocks=128, max_num_batched_tokens=512,
              max_num_seqs=16, max_model_len=256, enforce_eager=True)
    llm = LLM("tiny-moe", tensor_parallel_size=2, **kw)
    try:
        stages = llm.model_runner.init_stages
        assert {"device", "process_group", "model", "weights", "kv_cache", "total"} <= set(stages)
        out = capfd.readouterr().out
        assert "[init] rank 0 weights" in out and "[init] rank 1 ready" in out
        llm.model_runner.call("start_profiling")  # the reference's spelling reaches every rank
        llm.generate(_prompts(4), SamplingParams(temperature=0.0, max_tokens=4, ignore_eos=True), use_tqdm=False)
        snap = llm.profile_snapshot()
        llm.stop_profiling()
        assert llm.model_runner.call("memory_report")["rank"] == 0
        assert [r["rank"] for r in llm.executor.call_all("graph_report")] == [0, 1]
    finally:
        llm.exit()
    assert [s["rank"] for s in snap["ranks"]] == [0, 1]
    worst = snap["max_over_ranks"]
    assert worst["forward"]["count"] > 0 and worst["attn.core"]["p50_ms"] > 0
    for name, w in worst.items():
        assert w["p95_ms"] == max(s["segments"].get(name, {"p95_ms": 0.0})["p95_ms"] for s in snap["ranks"])
