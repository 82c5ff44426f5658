"""Online benchmark client against a real OpenAI server (tiny model on CPU) on a loopback port."""
import threading
import time

import pytest

from b200moe import bench_online
from b200moe.async_engine import AsyncLLMEngine
from b200moe.engine.executor import free_port
from b200moe.entrypoints.openai.api_server import create_app


@pytest.fixture(scope="module")
def server():
    import asyncio

    import uvicorn
    eng = AsyncLLMEngine("tiny-moe", device="cpu", kvcache_block_size=16, num_kvcache_blocks=512,
                         max_num_batched_tokens=1024, max_num_seqs=8, max_model_len=1024, enforce_eager=True)
    port = free_port()
    srv = uvicorn.Server(uvicorn.Config(create_app(eng, "tiny"), host="127.0.0.1", port=port, log_level="warning"))
    th = threading.Thread(target=srv.run, daemon=True)
    th.start()
    t0 = time.monotonic()
    while not srv.started:
        assert time.monotonic() - t0 < 60, "server did not start"
        time.sleep(0.05)
    try:
        yield f"http://127.0.0.1:{port}"
    finally:
        srv.should_exit = True
        th.join(timeout=30)
        asyncio.run(asyncio.wait_for(eng.close(), timeout=30))


def _args(base, out, *extra):
    return ["--base-url", base, "--model", "tiny", "--requests", "6", "--warmup-requests", "1", "--max-tokens", "5",
            "--prompt-words", "12", "--no-gpu-sample", "--output", str(out), *extra]


def test_poisson_points(server, tmp_path):
    p = bench_online.main(_args(server, tmp_path / "p.json", "--max-qps", "20", "--fractions", "0.5,1",
                                "--prompt-mode", "unique", "--prompt-words", "6", "--repeats", "2"))
    assert p["schema_version"] == 3 and len(p["points"]) == 4
    for s in p["points"]:
        assert s["counts"]["attempted"] == 6 and s["success_rate"] == 1.0
        assert s["output_tokens_per_s"] > 0 and s["ttft_p50_s"] is not None
        assert s["admission_counts"]["admitted"] == 6 and s["error_buckets"]["none"] == 6
        assert s["decode_steps"] + s["mixed_steps"] > 0  # /metrics scrape deltas
    assert len(p["aggregate"]) == 2 and p["aggregate"][0]["repeats"] == [1, 2]
    r = p["records"][0]
    assert r["done_received"] and r["output_tokens"] == 5 and len(r["itls_s"]) >= 1


def test_concurrency_shared_prefix(server, tmp_path):
    p = bench_online.main(_args(server, tmp_path / "c.json", "--concurrency", "2,4", "--prompt-mode", "shared",
                                "--prompt-words", "40"))
    assert [s["concurrency"] for s in p["points"]] == [2, 4]
    assert all(s["max_concurrency"] <= s["concurrency"] for s in p["points"])
    assert p["points"][1]["prefix_cache_hit_rate"] > 0  # shared prompts reuse full KV blocks


def test_unreachable_server_buckets_errors(tmp_path):
    port = free_port()
    args = bench_online.parse_args(_args(f"http://127.0.0.1:{port}", tmp_path / "x.json", "--warmup-requests", "0",
                                         "--concurrency", "2"))
    import asyncio
    p = asyncio.run(bench_online.async_main(args))
    s = p["points"][0]
    assert s["success_rate"] == 0.0 and s["error_buckets"]["stream"] == 6
    assert s["admission_counts"]["unknown"] == 6


def test_online_workload_token_prompts(server, tmp_path):
    """The online workload's shape at tiny scale: lognormal token-id prompts to
    /v1/completions, per-request output lengths decoded in full (ignore_eos),
    sampling at T 0.7 / top-p 0.9, and a cap on in-flight Poisson requests."""
    p = bench_online.main(_args(server, tmp_path / "o.json", "--workload", "online", "--max-qps", "50",
                                "--fractions", "1", "--prompt-median", "40", "--prompt-min", "16",
                                "--prompt-max", "64", "--prompt-vocab", "1000", "--output-len-range", "2,6",
                                "--max-concurrency", "2"))
    s = p["points"][0]
    assert s["success_rate"] == 1.0 and s["max_concurrency"] <= 2
    shape = bench_online.RequestShape(bench_online.parse_args(_args(server, "x", "--workload", "online",
                                                                    "--output-len-range", "2,6")))
    for r in p["records"]:
        assert 16 <= r["prompt_tokens"] <= 64
        assert r["output_tokens"] == shape.max_tokens(5, r["request_id"])  # ignore_eos: the drawn length
    lens = {r["prompt_tokens"] for r in p["records"]}
    assert len(lens) > 1
