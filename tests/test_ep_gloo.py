"""Expert-parallel plumbing on CPU: two gloo ranks (spawned by the engine),
data-parallel attention, experts split across ranks; tokens must match the
single-rank engine (fp32 tiny model)."""
import random

import numpy as np

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
