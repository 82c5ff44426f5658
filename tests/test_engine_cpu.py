"""End-to-end engine tests on CPU with the BASELINE tiny Qwen3-MoE (fp32)."""
import random

import numpy as np
import torch
import pytest

from b200moe import LLM, SamplingParams
from b200moe.models.reference import full_forward_logits


def _prompts(n=8, seed=0, lo=16, hi=64):
    rng = random.Random(seed)
    return [[rng.randrange(1024) for _ in range(rng.randint(lo, hi))] for _ in range(n)]


def _llm(**kw):
    base = dict(device="cpu", kvcache_block_size=16, num_kvcache_blocks=256, max_num_batched_tokens=1024,
                max_num_seqs=16, max_model_len=512, enforce_eager=True)
    base.update(kw)
    return LLM("tiny-moe", **base)


GREEDY = SamplingParams(temperature=0.0, max_tokens=32, ignore_eos=True)


@pytest.fixture(scope="module")
def baseline():
    llm = _llm()
    prompts = _prompts()
    out = [o["token_ids"] for o in llm.generate(prompts, GREEDY, use_tqdm=False)]
    yield llm, prompts, out
    llm.exit()


def test_tokens_match_full_recompute_oracle(baseline):
    llm, prompts, out = baseline
    model = llm.model_runner.model
    total = mismatch = 0
    for p, toks in zip(prompts, out):
        logits = full_forward_logits(model, p + toks)
        pred = logits[len(p) - 1:len(p) + len(toks) - 1]
        for j, t in enumerate(toks):
            total += 1
            top2 = pred[j].topk(2).values
            if int(pred[j].argmax()) != t:
                mismatch += 1
                # a flip is only acceptable at a near-tie: bf16 rounding of the router
                # logits (the reference's routing numerics) is discontinuous, so fp32
                # reordering upstream can move a logit across a rounding boundary
                assert float(top2[0] - pred[j][t]) < 5e-3
    assert mismatch <= 0.03 * total


def test_overlap_pipeline_bitwise_equal(baseline):
    _, prompts, out = baseline
    llm = _llm(scheduler_overlap=True)
    res = [o["token_ids"] for o in llm.generate(prompts, GREEDY, use_tqdm=False)]
    llm.exit()
    assert res == out


def test_stall_free_chunked_prefill(baseline):
    _, prompts, out = baseline
    llm = _llm(scheduler_policy="stall_free", prefill_chunk_size=16, max_num_batched_tokens=64)
    res = [o["token_ids"] for o in llm.generate(prompts, GREEDY, use_tqdm=False)]
    m = llm.metrics()
    llm.exit()
    assert m.get("engine_mixed_steps_total", 0) > 0
    agree = np.mean([a == b for ra, rb in zip(res, out) for a, b in zip(ra, rb)])
    assert agree > 0.98


def test_prefix_cache_hits_and_same_tokens(baseline):
    _, prompts, out = baseline
    llm = _llm(kvcache_block_size=16)
    shared = [list(range(100, 148)) + p for p in prompts[:4]]
    a = [o["token_ids"] for o in llm.generate(shared, GREEDY, use_tqdm=False)]
    hit0 = llm.metrics()["kv_prefix_hit_tokens_total"]
    b = [o["token_ids"] for o in llm.generate(shared, GREEDY, use_tqdm=False)]
    hit1 = llm.metrics()["kv_prefix_hit_tokens_total"]
    llm.exit()
    # prompts admitted in the same step cannot hit each other (hashes are
    # registered after the step); the second pass hits the first pass's blocks
    assert hit1 > hit0
    agree = np.mean([x == y for ra, rb in zip(a, b) for x, y in zip(ra, rb)])
    assert agree > 0.98


def test_preemption_under_kv_pressure(baseline):
    _, prompts, out = baseline
    llm = _llm(num_kvcache_blocks=16)
    res = [o["token_ids"] for o in llm.generate(prompts, GREEDY, use_tqdm=False)]
    m = llm.metrics()
    llm.exit()
    assert m["scheduler_preemptions_total"] > 0
    agree = np.mean([a == b for ra, rb in zip(res, out) for a, b in zip(ra, rb)])
    assert agree > 0.98


def test_generate_returns_text_tokens_metrics(baseline):
    llm, prompts, _ = baseline
    outs = llm.generate(["hello world"], SamplingParams(temperature=0.0, max_tokens=4, ignore_eos=True),
                        use_tqdm=False)
    o = outs[0]
    assert set(o) == {"text", "token_ids", "metrics"}
    assert len(o["token_ids"]) == 4 and isinstance(o["text"], str)
    for key in ("prompt_tokens", "output_tokens", "ttft_s", "tpot_s", "e2e_s", "itls_s", "finish_reason"):
        assert key in o["metrics"]
    assert o["metrics"]["finish_reason"] == "length"


def test_admission_checks(baseline):
    llm = baseline[0]
    with pytest.raises(ValueError):
        llm.add_request([5000], SamplingParams(max_tokens=4))          # out of vocab
    with pytest.raises(ValueError):
        llm.add_request([1] * 500, SamplingParams(max_tokens=100))    # > max_model_len
    small = _llm(num_kvcache_blocks=4, max_model_len=512)
    with pytest.raises(OverflowError):
        small.add_request([1] * 100, SamplingParams(max_tokens=10))  # > KV capacity (64 tokens)
    small.exit()


def test_stop_tokens_and_sampling_cpu(baseline):
    llm, prompts, out = baseline
    stop = out[0][5]
    res = llm.generate([prompts[0]], SamplingParams(temperature=0.0, max_tokens=32, stop_token_ids=[stop]),
                       use_tqdm=False)[0]
    assert res["token_ids"][-1] == stop and res["metrics"]["finish_reason"] == "stop"
    sp = SamplingParams(temperature=0.8, top_k=20, top_p=0.9, max_tokens=8, seed=7)
    a = llm.generate(prompts[:2], sp, use_tqdm=False)
    b = llm.generate(prompts[:2], sp, use_tqdm=False)
    assert [o["token_ids"] for o in a] == [o["token_ids"] for o in b]


def test_tile_major_fp8_layout_roundtrip():
    """tile_fp8 puts each (128-row, 64-K) block of an e4m3 matrix in one
    contiguous 8 KB run; untile_fp8 inverts it, and the CPU linear path reads
    either layout to the same result."""
    import torch
    from b200moe import ops
    from b200moe.utils.weights import quantize_block_fp8
    w = torch.randn(3, 256, 384) * 0.05
    q = torch.stack([quantize_block_fp8(w[i])[0] for i in range(3)])
    t = ops.tile_fp8(q)
    assert t.shape == q.shape
    # block (expert 1, row tile 1, K stage 2) is one contiguous 8 KB run; chunk u of
    # row r sits at chunk u ^ ((r >> 1) & 3) (the 64-byte swizzle the GEMM reads)
    blk = t[1].view(torch.uint8).reshape(-1)[(1 * (384 // 64) + 2) * 8192:(1 * (384 // 64) + 3) * 8192]
    blk = blk.view(128, 4, 16)
    want = q[1, 128:256, 128:192].contiguous().view(torch.uint8).view(128, 4, 16)
    for r in (0, 1, 2, 5, 77, 127):
        for u in range(4):
            assert torch.equal(blk[r, u ^ ((r >> 1) & 3)], want[r, u])
    assert torch.equal(ops.untile_fp8(t).view(torch.uint8), q.view(torch.uint8))
    s = quantize_block_fp8(w[0])[1]
    x = torch.randn(5, 384).to(torch.bfloat16)
    assert torch.equal(ops.linear(x, q[0], s), ops.linear(x, t[0], s, tiled=True))


def test_dense_planner_splits_are_valid_for_wide_stages():
    """plan_dense picks K splits in units of the stage width the kernel will use
    (128-wide stages for e4m3 tiles of <= 128 tokens): no split is ever empty."""
    import math
    from b200moe import ops
    for rows in (1, 7, 64, 256, 300, 1024):
        for n, k in ((5120, 2048), (2048, 4096), (2048, 768), (256, 256)):
            bn, splits = ops.plan_dense(rows, n // 128, k // 64)
            stages = k // 128 if bn <= 128 else k // 64
            per = math.ceil(stages / splits)
            assert (splits - 1) * per < stages, (rows, n, k, bn, splits)


def test_dequant_weights_cpu_matches_block_dequant():
    """ops.dequant_weights (row-major or tile-major e4m3 input) equals
    bf16(float(q) * block scale) per expert."""
    import torch
    from b200moe import ops
    from b200moe.utils.weights import quantize_block_fp8
    w = torch.randn(2, 256, 384) * 0.05
    qs = [quantize_block_fp8(w[i]) for i in range(2)]
    q = torch.stack([a for a, _ in qs])
    s = torch.stack([b for _, b in qs])
    want = torch.stack([ops.dequant_block_fp8(q[i], s[i]) for i in range(2)]).to(torch.bfloat16)
    for tiled in (False, True):
        out = torch.empty(2, 256, 384, dtype=torch.bfloat16)
        ops.dequant_weights(ops.tile_fp8(q) if tiled else q, s, out, tiled)
        assert torch.equal(out, want)


def test_natural_layout_restores_tiling():
    """Loaders run on the row-major layout and the tile-major layout comes back after."""
    from b200moe.utils.weights import natural_layout

    class Fake:
        def __init__(self):
            self.weights_tiled = True
            self.calls = []

        def untile_weights_(self):
            self.calls.append("untile")
            self.weights_tiled = False

        def tile_weights_(self):
            self.calls.append("tile")
            self.weights_tiled = True

    m = Fake()
    with natural_layout(m):
        assert not m.weights_tiled
    assert m.weights_tiled and m.calls == ["untile", "tile"]
    m2 = Fake()
    m2.weights_tiled = False
    with natural_layout(m2):
        pass
    assert m2.calls == []


def test_launch_ahead_decode_matches_plain_steps():
    """Decode steps launched before the previous step's tokens are read back
    (their input token read on the device) give the tokens of plain stepping,
    with sequences finishing at different steps (length limits and stop tokens)."""
    import random as _r
    rng = _r.Random(3)
    prompts = [[rng.randrange(1, 400) for _ in range(rng.randrange(5, 60))] for _ in range(7)]
    sps = [SamplingParams(temperature=0.0, max_tokens=rng.randrange(1, 25), ignore_eos=bool(i % 2),
                          stop_token_ids=[rng.randrange(1, 400)]) for i in range(len(prompts))]
    base = dict(kvcache_block_size=16, max_num_seqs=8, max_num_batched_tokens=256, max_model_len=256,
                num_kvcache_blocks=128, device="cpu", enforce_eager=True)
    ahead = LLM("tiny-moe-fp8", scheduler_overlap=True, **base)
    plain = LLM("tiny-moe-fp8", scheduler_overlap=False, **base)
    a = ahead.generate(prompts, sps, use_tqdm=False)
    b = plain.generate(prompts, sps, use_tqdm=False)
    assert [x["token_ids"] for x in a] == [x["token_ids"] for x in b]
    assert ahead.metrics()["engine_decode_feed_steps_total"] > 0


def test_plan_validation_rejects_out_of_range_indices():
    """The host check in front of every launch: block ids, KV slots, token ids,
    feed rows and context lengths outside their buffers raise before any
    kernel sees them; the engine's own plans pass it."""
    from b200moe.engine.sequence import Sequence
    from b200moe.engine.step_plan import build_plan, validate_plan
    Sequence.block_size = 16
    s = Sequence(list(range(40)), SamplingParams(max_tokens=4))
    s.block_table = [3, 5, 7]
    plan = build_plan([s], [40], [True], 16, max_blocks=4)
    validate_plan(plan, num_blocks=8, block_size=16, vocab=1000, feed_rows=8)
    for field, value, msg in (("block_tables", 8, "block id"), ("slot_mapping", 8 * 16, "KV slot"),
                              ("input_ids", 1000, "token id"), ("seq_lens", 65, "context length")):
        bad = build_plan([s], [40], [True], 16, max_blocks=4)
        getattr(bad, field).reshape(-1)[0] = value
        with pytest.raises(ValueError, match=msg):
            validate_plan(bad, num_blocks=8, block_size=16, vocab=1000, feed_rows=8)
    s2 = Sequence(list(range(20)), SamplingParams(max_tokens=4))
    s2.block_table = [1, 2]
    s2.cached_len = 19
    fed = build_plan([s2], [1], [False], 16, max_blocks=4, feed={id(s2): 9})
    with pytest.raises(ValueError, match="feed row"):
        validate_plan(fed, num_blocks=8, block_size=16, vocab=1000, feed_rows=8)
    llm = LLM("tiny-moe", device="cpu", kvcache_block_size=16, num_kvcache_blocks=8, max_num_batched_tokens=128,
              max_num_seqs=4, max_model_len=64, enforce_eager=True)
    try:
        plan.block_tables[0, 0] = 8 + 1  # the runner's pool has 8 blocks (+ its scratch block)
        with pytest.raises(ValueError, match="block id"):
            llm.model_runner.launch(plan)
        assert not llm.model_runner._pending
        out = llm.generate([[1, 2, 3]], SamplingParams(temperature=0.0, max_tokens=3, ignore_eos=True),
                           use_tqdm=False)
        assert len(out[0]["token_ids"]) == 3
    finally:
        llm.exit()


def test_per_step_jsonl_trace(tmp_path):
    """``metrics_path``: one JSON line per step with mode, batch, token counts,
    query / context lengths and schedule / forward seconds
    (reference: nanovllm/engine/llm_engine.py:459-474)."""
    import json
    path = tmp_path / "steps.jsonl"
    llm = LLM("tiny-moe", device="cpu", kvcache_block_size=16, num_kvcache_blocks=32, max_num_batched_tokens=128,
              max_num_seqs=4, max_model_len=128, enforce_eager=True, metrics_path=str(path))
    try:
        llm.generate([[1, 2, 3, 4], list(range(10, 40))],
                     SamplingParams(temperature=0.0, max_tokens=3, ignore_eos=True), use_tqdm=False)
    finally:
        llm.exit()
    recs = [json.loads(line) for line in path.read_text().splitlines()]
    assert recs and all(r["kind"] == "step" for r in recs)
    assert recs[0]["mode"] == "prefill" and recs[0]["prefill_tokens"] == 34 and recs[0]["query_lens"] == [4, 30]
    assert recs[-1]["mode"] == "decode" and recs[-1]["decode_tokens"] == 2
    assert sum(r["prefill_tokens"] for r in recs) == 34 and sum(r["decode_tokens"] for r in recs) == 4
    assert all(r["forward_s"] >= 0 and r["schedule_s"] >= 0 for r in recs)


def test_overlap_toggled_mid_run_drains_and_matches():
    """Overlap switched off and on again while requests are in flight (on ->
    off -> on): the parked and launched steps drain without losing or
    repeating a token, and the outputs equal a run without overlap."""
    import random as _r
    rng = _r.Random(5)
    prompts = [[rng.randrange(1, 400) for _ in range(rng.randrange(5, 50))] for _ in range(6)]
    sps = [SamplingParams(temperature=0.0, max_tokens=rng.randrange(4, 30), ignore_eos=True) for _ in prompts]
    base = dict(kvcache_block_size=16, max_num_seqs=8, max_num_batched_tokens=256, max_model_len=256,
                num_kvcache_blocks=128, device="cpu", enforce_eager=True)
    plain = LLM("tiny-moe-fp8", scheduler_overlap=False, **base)
    want = [o["token_ids"] for o in plain.generate(prompts, sps, use_tqdm=False)]
    plain.exit()
    eng = LLM("tiny-moe-fp8", scheduler_overlap=True, **base)
    try:
        ids = [eng.add_request(p, sp) for p, sp in zip(prompts, sps)]
        got, steps = {}, 0
        while not eng.is_finished():
            steps += 1
            assert steps < 500
            if steps == 4:
                eng.set_scheduler_overlap(False)
            if steps == 9:
                eng.set_scheduler_overlap(True)
            out, _ = eng.step()
            for sid, toks, _m in out:
                assert sid not in got, "a request finished twice"
                got[sid] = toks
        assert [got[i] for i in ids] == want
    finally:
        eng.exit()


def test_logprobs_and_penalties_through_engine_cpu():
    """Log-probs ride each step's token read-back: greedy rows report their token as
    the top entry with the chosen log-prob equal to it; a sampled row with every
    filter and penalty reports sorted top entries that bound its chosen log-prob."""
    from b200moe.engine.llm_engine import LLMEngine
    eng = LLMEngine("tiny-moe", device="cpu", kvcache_block_size=16, num_kvcache_blocks=64,
                    max_num_batched_tokens=256, max_num_seqs=8, max_model_len=256, enforce_eager=True)
    try:
        a = eng.add_request(list(range(5, 25)), SamplingParams(temperature=0.0, max_tokens=5, ignore_eos=True,
                                                               logprobs=4))
        b = eng.add_request(list(range(30, 50)), SamplingParams(
            temperature=0.9, top_k=40, top_p=0.9, min_p=0.02, max_tokens=5, ignore_eos=True, logprobs=2, seed=3,
            repetition_penalty=1.2, presence_penalty=0.4, frequency_penalty=0.1))
        events = {a: [], b: []}
        while not eng.is_finished():
            eng.step()
            for sid, tok, _, _, lp in eng.last_token_events:
                events[sid].append((tok, lp))
        assert len(events[a]) == 5 and len(events[b]) == 5
        for tok, lp in events[a]:
            assert len(lp["top"]) >= 4 and lp["top"][0][0] == tok
            assert abs(lp["top"][0][1] - lp["chosen"]) < 1e-5
            vals = [v for _, v in lp["top"]]
            assert vals == sorted(vals, reverse=True) and vals[0] <= 0.0
        for tok, lp in events[b]:
            vals = [v for _, v in lp["top"]]
            assert vals == sorted(vals, reverse=True) and lp["chosen"] <= vals[0] + 1e-6 and lp["chosen"] <= 0.0
    finally:
        eng.exit()


def test_int8_channel_kv_store_gather_and_calibration_cpu():
    """The reference's int8 channel mode on the CPU path: calibration finds a planted
    outlier channel (amax / mean |x| > 10), which then round-trips exactly through
    the bf16 side pool while the other channels come back within half a quantum."""
    from b200moe.engine.kv_cache import KVPool, NOUT_MAX
    g = torch.Generator().manual_seed(0)
    H, D, bs = 2, 64, 16
    pool = KVPool(9, 1, H, bs, D, torch.bfloat16, "cpu", int8=True, int8_mode="channel")
    layer = pool.layer(0)
    k = torch.randn(40, H, D, generator=g)
    v = torch.randn(40, H, D, generator=g)
    k[3, 1, 5] = 80.0               # one rare large value: an outlier channel of K, head 1
    slots = torch.arange(40, dtype=torch.int32)
    pool.calibrate_begin()
    layer.store(slots, k.to(torch.bfloat16), v.to(torch.bfloat16))
    n = pool.calibrate_freeze(tokens_seen=40)
    assert n >= 1 and int(pool.n_out[0, 1]) >= 1 and 5 in pool.out_idx[0, 1].tolist()
    assert pool.n_out.max() <= NOUT_MAX and float(pool.ch_dscale[0, 0, 1, 5]) == 0.0
    layer.store(slots, k.to(torch.bfloat16), v.to(torch.bfloat16))
    kk, vv = layer.gather(torch.arange(3), 40)
    kb = k.to(torch.bfloat16).float()
    assert torch.equal(kk[:, 1, 5].float(), kb[:, 1, 5])      # the outlier channel is exact
    step = pool.ch_scale[0, 0]                                # [H, D] quantum of K
    err = (kk.float() - kb).abs()
    assert (err <= step * 0.5 + 1e-2 * kb.abs() + 1e-6).all()


def test_int8_channel_kv_engine_cpu():
    """An engine in int8 channel mode calibrates at start-up and then generates."""
    llm = LLM("tiny-moe", device="cpu", kvcache_block_size=16, num_kvcache_blocks=128, max_num_batched_tokens=512,
              max_num_seqs=8, max_model_len=512, enforce_eager=True, kv_cache_dtype="int8", kv_int8_mode="channel")
    try:
        assert llm.kv_outlier_dims is not None
        assert float(llm.model_runner.kv.ch_scale.max()) != 1.0 / 127.0  # frozen from real statistics
        out = llm.generate([[5, 6, 7, 8, 9], list(range(30, 70))],
                           SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True), use_tqdm=False)
        assert all(len(o["token_ids"]) == 6 for o in out)
    finally:
        llm.exit()


def test_resident_bf16_expert_copy_decision(monkeypatch):
    """The resident bf16 expert copy is kept only on CUDA, for the single-GPU or fused
    expert-parallel paths, and only when enough memory stays free for the KV cache
    ("auto"); "1" forces it and "0" turns it off."""
    from types import SimpleNamespace
    from b200moe.engine.model_runner import ModelRunner
    GiB = 1 << 30
    calls = []

    def model(ep=None, need=60 * GiB):
        return SimpleNamespace(ep=ep, attn_tp=1, BF16_EXPERT_ROWS=512, bf16_expert_bytes=lambda: need,
                               cache_bf16_experts_=lambda: calls.append(1) or need)

    def decide(m, free, mode="auto", dev="cuda"):
        monkeypatch.setenv("B200MOE_BF16_EXPERT_CACHE", mode)
        monkeypatch.setattr(torch.cuda, "mem_get_info", lambda d=None: (free, 180 * GiB))
        runner = SimpleNamespace(model=m, device=torch.device(dev), BF16_CACHE_KEEP_FREE=0.35)
        return ModelRunner._maybe_cache_bf16_experts(runner)

    assert decide(model(), free=150 * GiB) == 60 * GiB                 # 90 GiB stay free: keep it
    assert decide(model(), free=100 * GiB) == 0                        # 40 GiB would stay: no
    assert decide(model(), free=100 * GiB, mode="1") == 60 * GiB       # forced
    assert decide(model(), free=150 * GiB, mode="0") == 0              # off
    assert decide(model(), free=150 * GiB, dev="cpu") == 0             # CUDA only
    assert decide(model(ep=SimpleNamespace(backend="nccl_a2a")), free=150 * GiB) == 0
    assert decide(model(ep=SimpleNamespace(backend="fused")), free=150 * GiB) == 60 * GiB
    assert len(calls) == 3
