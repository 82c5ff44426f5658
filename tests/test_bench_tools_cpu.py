"""Benchmark tooling on CPU: metric library, offline driver (gate + sweep), tiny checkpoint generator."""
import json
import math

import pytest

from b200moe import benchmarking as bm


# ----------------------------------------------------------- metric library
def test_wilson_ci():
    lo, hi = bm.wilson_ci(128, 128)
    assert lo == pytest.approx(0.971, abs=0.002) and hi == pytest.approx(1.0, abs=0.002)
    assert bm.wilson_ci(0, 0) == (None, None)
    lo, hi = bm.wilson_ci(0, 128)
    assert lo == 0.0 and hi < 0.03
    lo, hi = bm.wilson_ci(50, 100)
    assert lo == pytest.approx(0.4038, abs=1e-3) and hi == pytest.approx(0.5962, abs=1e-3)


def test_percentiles():
    assert bm.percentile([0, 10], 0.95, method="linear") == pytest.approx(9.5)
    assert bm.percentile([0, 10], 0.95) == 10
    assert bm.percentile([None, 3, 1, 2], 0.5) == 2
    assert bm.percentile([], 0.5) is None
    with pytest.raises(ValueError):
        bm.percentile([1], 1.5)
    d = bm.distribution([0.1, 0.2, 0.3, None], "ttft")
    assert d == {"ttft_p50_s": 0.2, "ttft_p95_s": 0.3, "ttft_p99_s": 0.3}


def test_tpot_cv_goodput():
    assert bm.request_tpot(1.1, 0.1, 11) == pytest.approx(0.1)
    assert bm.request_tpot(1.0, 0.1, 1) is None
    assert bm.coefficient_of_variation([1.0]) == 0.0
    assert bm.coefficient_of_variation([0.0, 0.0]) == 0.0
    assert bm.coefficient_of_variation([2.0, 4.0]) == pytest.approx(math.sqrt(2) / 3)
    rows = [{"ok": True, "ttft_s": 0.5, "tpot_s": 0.1}, {"ok": True, "ttft_s": 3.0, "tpot_s": 0.1},
            {"ok": False, "ttft_s": None, "tpot_s": None}]
    assert bm.goodput(rows, 2.0, 2.0, 0.5) == pytest.approx(0.5)
    recs = [{"output_tokens": 64, "conforming_standard": i < 100} for i in range(128)]
    assert bm.token_goodput(recs, 100.0) == pytest.approx(64.0)
    assert bm.token_goodput(recs, 0.0) == 0.0


def test_dual_slo_and_errors():
    stall = {"ok": True, "ttft_s": 0.5, "tpot_s": 0.2, "itls_s": [0.1] * 20 + [2.0]}
    assert bm.conforming(stall, 2.0, 0.5) == (True, False)
    assert bm.conforming({**stall, "itls_s": [0.1] * 20}, 2.0, 0.5) == (True, True)
    assert bm.conforming({"ok": False, "ttft_s": None, "tpot_s": None}, 2.0, 0.5) == (False, False)
    assert bm.max_itl_s(stall) == 2.0
    rows = [{"ok": False, "timed_out": True}, {"ok": False, "http_status": 500},
            {"ok": False, "error": "stream ended before [DONE]"},
            {"ok": False, "error": "token usage missing and no local tokenizer"},
            {"ok": False, "http_status": 429}, {"ok": True}]
    c = bm.error_bucket_counts(rows)
    assert c == {"none": 1, "timeout": 1, "http": 1, "reject_429": 1, "stream": 1, "token_count": 1}


# ---------------------------------------------------------- offline driver
def test_offline_driver_gate_and_sweep(tmp_path):
    from b200moe import bench_offline
    common = ["--model", "tiny-moe", "--device", "cpu", "--random-init", "--enforce-eager",
              "--kvcache-block-size", "16", "--max-num-batched-tokens", "512", "--prompt-len", "40",
              "--output-len", "4", "--repeats", "2", "--verify-max-tokens", "3", "--verify-repeats", "2"]
    ref = tmp_path / "ref.json"
    out1 = tmp_path / "a.json"
    p1 = bench_offline.main(common + ["--batches", "1,3", "--moe-backends", "fused,loop",
                                      "--verify-backends", "fused,loop", "--freeze-reference", str(ref),
                                      "--output", str(out1)])
    assert p1["verification"]["passed"] and ref.is_file()
    assert len(json.loads(ref.read_text())) == 4
    assert len(p1["records"]) == 2 * 2 * 2  # backends x batches x repeats
    assert {s["batch"] for s in p1["summary"]} == {1, 3}
    assert all(r["output_tokens"] == r["batch"] * 4 for r in p1["records"])
    jsonl = out1.with_suffix(".jsonl").read_text().strip().splitlines()
    assert len(jsonl) == len(p1["records"])
    # frozen reference gate + prefix-cache cold/hot probe
    p2 = bench_offline.main(common + ["--batches", "2", "--reference-outputs", str(ref), "--cache-modes", "cold,hot",
                                      "--shared-prefix-len", "32", "--probe-batches", "2",
                                      "--probe-prompt-len", "48", "--probe-shared-prefix-len", "32",
                                      "--output", str(tmp_path / "b.json")])
    assert all(p2["verification"]["backends"]["fused"]["reference_matches"])
    hot = [r for r in p2["records"] if r["phase"] == "matrix" and r["cache_mode"] == "hot"]
    cold = [r for r in p2["records"] if r["phase"] == "matrix" and r["cache_mode"] == "cold"]
    hit = lambda r: r["cache_metrics_delta"]["kv_prefix_hit_tokens_total"]
    assert sum(hit(r) for r in hot) > sum(hit(r) for r in cold)
    assert p2["provenance"]["reference_sha256"]


def test_offline_driver_rejects_bad_reference(tmp_path):
    from b200moe import bench_offline
    bad = tmp_path / "bad.json"
    bad.write_text(json.dumps([{"token_ids": [1, 2, 3]}] * 4))
    with pytest.raises(SystemExit, match="frozen reference mismatch"):
        bench_offline.main(["--model", "tiny-moe", "--device", "cpu", "--random-init", "--enforce-eager",
                            "--kvcache-block-size", "16", "--max-num-batched-tokens", "256", "--batches", "1",
                            "--prompt-len", "8", "--output-len", "2", "--repeats", "1", "--verify-max-tokens", "3",
                            "--verify-repeats", "1", "--reference-outputs", str(bad),
                            "--output", str(tmp_path / "x.json")])


# ------------------------------------------------------- tiny checkpoint
def test_make_tiny_moe_roundtrip(tmp_path):
    from b200moe import LLM, SamplingParams
    from b200moe.utils.make_tiny_moe import tiny_config, tiny_state, write_tiny_moe
    a, b = tiny_state(tiny_config(), 0), tiny_state(tiny_config(), 0)
    assert all((a[k] == b[k]).all() for k in a)
    assert len(a) == 3 + 2 * (9 + 8 * 3)
    path = write_tiny_moe(str(tmp_path / "tiny"))
    cfg = json.loads((tmp_path / "tiny" / "config.json").read_text())
    assert (cfg["hidden_size"], cfg["head_dim"], cfg["num_experts"], cfg["vocab_size"]) == (64, 16, 8, 151936)
    llm = LLM(path, device="cpu", enforce_eager=True, kvcache_block_size=16, num_kvcache_blocks=32,
              max_num_batched_tokens=128, max_num_seqs=2, max_model_len=128)
    try:
        out = llm.generate([[1, 2, 3], "<7> <8>"], SamplingParams(temperature=0.0, max_tokens=3, ignore_eos=True),
                           use_tqdm=False)
        assert [len(o["token_ids"]) for o in out] == [3, 3]
    finally:
        llm.exit()


# ------------------------------------------------------------- charts
def test_svg_charts(tmp_path):
    import xml.etree.ElementTree as ET
    from b200moe import charts
    off = tmp_path / "off.json"
    off.write_text(json.dumps({"summary": [
        {"phase": "matrix", "backend": b, "attention_backend": "paged", "batch": n, "throughput_median": t}
        for b, f in (("fused", 1.0), ("loop", 0.5)) for n, t in ((1, 100 * f), (8, 700 * f), (64, 3000 * f))]}))
    onl = tmp_path / "on.json"
    onl.write_text(json.dumps({"points": [{"achieved_qps": q, "slo_standard_rate": r, "slo_strict_rate": r * 0.9,
                                           "tpot_p95_s": 0.05 * q} for q, r in ((1, 1.0), (2, 1.0), (4, 0.7))]}))
    bl = tmp_path / "bench.jsonl"
    bl.write_text("\n".join(json.dumps({"value": 9000.0 * n, "n_gpus": n, "unit": "tok/s"}) for n in (1, 2, 4, 8)))
    mic = tmp_path / "micro.jsonl"
    mic.write_text('{"kernel": "moe_gate_up_silu", "hbm_frac": 0.52, "tc_frac": 0.06, "tokens": 256}\nmicro rc=0\n')
    files = charts.render(str(tmp_path / "charts"), off, onl, bl, mic)
    assert len(files) == 4
    for f in files:
        root = ET.parse(f).getroot()  # well-formed SVG
        assert root.tag.endswith("svg")
        assert "sha256" in open(f).read()
    assert open(files[0]).read().count("<polyline") == 2


def test_offline_driver_workload_presets():
    """Named workloads fill in the model and shapes; explicit flags win; the
    KV options reach the engine's keyword arguments."""
    from b200moe.bench_offline import engine_kwargs, parse_args
    a = parse_args(["--workload", "longctx", "--kv-offload", "--num-kvcache-blocks", "600", "--random-init",
                    "--skip-verification"])
    assert (a.model, a.batches, a.prompt_len, a.output_len, a.kvcache_block_size) == \
        ("qwen3-30b-a3b", "8", 32768, 512, 256)
    kw = engine_kwargs(a)
    assert kw["kv_cache_dtype"] == "bf16" and kw["kv_offload_enabled"] and kw["num_kvcache_blocks"] == 600
    assert kw["max_model_len"] == 32768 + 512 + 16 and kw["max_num_seqs"] == 8
    assert engine_kwargs(parse_args(["--workload", "longctx", "--kv-cache-dtype", "int8"]))["kv_cache_dtype"] == "int8"
    b = parse_args(["--workload", "235b", "--batches", "4", "--output-len", "32"])
    assert (b.model, b.batches, b.prompt_len, b.output_len) == ("qwen3-235b-a22b", "4", 2048, 32)
    kw = engine_kwargs(b)
    assert "kv_offload_enabled" not in kw and kw["kv_cache_dtype"] == "bf16" and kw["attention_parallel"] == "dp"
    c = parse_args([])
    assert c.model == "qwen3-30b-a3b" and c.prompt_len == 128


def test_bench_layout_label_follows_the_engine_report():
    """bench.py names the layout the engine reports (rank 0's parallel_report), not the flags."""
    import importlib.util
    import pathlib
    spec = importlib.util.spec_from_file_location("bench_main", pathlib.Path(__file__).resolve().parents[1] / "bench.py")
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    assert bench._parallelism(8, {"attention_parallel": "dp", "ep_backend": "fused"}) == "ep8+dp8-attn"
    assert bench._parallelism(2, {"attention_parallel": "tp", "tp_fused": True}) == "tp2-fused-peer-sums"
    assert bench._parallelism(2, {"attention_parallel": "tp", "tp_fused": False}) == "tp2-nccl"
    assert bench._parallelism(1, {"attention_parallel": "dp", "ep_backend": None}) == "ep1+dp1-attn"
