"""OpenAI server contract on CPU: a fake engine for the HTTP contract, and the
real async engine (tiny model on CPU) end to end."""
import asyncio
import json
from queue import Queue

import pytest
from fastapi.testclient import TestClient

from b200moe.async_engine import AsyncLLMEngine, RequestHandle, TokenEvent
from b200moe.entrypoints.openai.api_server import build_parser, create_app, is_loopback, main
from b200moe.utils.tokenizer import ByteTokenizer


class FakeEngine:
    """Emits the prompt's bytes back as tokens (echo model)."""

    def __init__(self, reject=None, error=False):
        self.tokenizer = ByteTokenizer(1024, 1023)
        self.reject = reject
        self.error = error
        self.cancelled = []
        self.last_sp = None
        self._id = 0

    async def add_request(self, prompt, sp):
        if self.reject:
            raise self.reject
        self.last_sp = sp
        q = Queue()
        toks = list(b"hello world!")[:sp.max_tokens]
        for i, t in enumerate(toks):
            last = i == len(toks) - 1
            if self.error and i == 2:
                q.put(TokenEvent(finished=True, error="boom"))
                break
            q.put(TokenEvent(token_id=t, finished=last,
                             metrics={"finish_reason": "length", "prompt_tokens": len(prompt),
                                      "output_tokens": len(toks), "ttft_s": 0.01} if last else None,
                             logprobs={"top": [(t, -0.1)], "chosen": -0.1} if sp.logprobs else None))
        self._id += 1
        return RequestHandle(self._id, q)

    async def next_event(self, h):
        return h.events.get()

    def cancel(self, seq_id):
        self.cancelled.append(seq_id)

    async def close(self):
        pass

    def prometheus_text(self):
        return "b200moe_requests_total 0\n"


def client(engine, **kw):
    return TestClient(create_app(engine, "tiny", **kw))


def test_health_models_metrics():
    c = client(FakeEngine())
    assert c.get("/health").json()["status"] == "ok"
    assert c.get("/v1/models").json()["data"][0]["id"] == "tiny"
    assert "b200moe_requests_total" in c.get("/metrics").text


def test_completion_non_stream_and_usage():
    e = FakeEngine()
    r = client(e).post("/v1/completions", json={"prompt": "abc", "max_tokens": 5, "temperature": 0})
    assert r.status_code == 200
    d = r.json()
    assert d["object"] == "text_completion" and d["choices"][0]["text"] == "hello"
    assert d["usage"] == {"prompt_tokens": 3, "completion_tokens": 5, "total_tokens": 8}


def test_chat_stream_sse_with_usage_and_metrics():
    body = {"messages": [{"role": "user", "content": "hi"}], "max_tokens": 12, "stream": True,
            "stream_options": {"include_usage": True, "include_metrics": True}}
    r = client(FakeEngine()).post("/v1/chat/completions", json=body)
    lines = [l for l in r.text.split("\n\n") if l]
    assert lines[-1] == "data: [DONE]"
    chunks = [json.loads(l[6:]) for l in lines[:-1]]
    text = "".join(c["choices"][0]["delta"].get("content", "") for c in chunks if c["choices"])
    assert text == "hello world!"
    final = [c for c in chunks if c["choices"] and c["choices"][0]["finish_reason"]][0]
    assert final["choices"][0]["finish_reason"] == "length" and "metrics" in final
    assert chunks[-1]["usage"]["completion_tokens"] == 12


def test_stop_string_retracted():
    r = client(FakeEngine()).post("/v1/completions", json={"prompt": "x", "max_tokens": 12, "stop": " wor"})
    d = r.json()
    assert d["choices"][0]["text"] == "hello" and d["choices"][0]["finish_reason"] == "stop"


def test_logprobs_shapes():
    c = client(FakeEngine())
    d = c.post("/v1/completions", json={"prompt": "x", "max_tokens": 3, "logprobs": 1}).json()
    lp = d["choices"][0]["logprobs"]
    assert set(lp) == {"tokens", "token_logprobs", "top_logprobs", "text_offset"} and len(lp["tokens"]) == 3
    d = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "x"}], "max_tokens": 3,
                                             "logprobs": True, "top_logprobs": 1}).json()
    assert len(d["choices"][0]["logprobs"]["content"]) == 3


@pytest.mark.parametrize("body,code", [
    ({"prompt": "x", "n": 2}, 400),
    ({"prompt": "x", "max_tokens": 0}, 400),
    ({"prompt": "x", "temperature": -1}, 400),
    ({"prompt": "x", "top_p": 0}, 400),
    ({"prompt": "x", "top_k": 0}, 400),
    ({"prompt": "x", "logprobs": 99}, 400),
    ({"prompt": "x", "stop": 5}, 400),
    ({"prompt": "x", "stop_token_ids": ["a"]}, 400),
    ({"prompt": "x", "response_format": {"type": "text"}}, 400),
    ({"prompt": 5}, 400),
    ({"prompt": "x", "echo": True}, 400),
])
def test_bad_requests(body, code):
    assert client(FakeEngine()).post("/v1/completions", json=body).status_code == code


def test_queue_full_is_429_and_value_error_400():
    assert client(FakeEngine(reject=OverflowError("full"))).post(
        "/v1/completions", json={"prompt": "x"}).status_code == 429
    assert client(FakeEngine(reject=ValueError("too long"))).post(
        "/v1/completions", json={"prompt": "x"}).status_code == 400


def test_engine_error_is_500_non_stream():
    r = client(FakeEngine(error=True)).post("/v1/completions", json={"prompt": "x", "max_tokens": 12})
    assert r.status_code == 500


def test_api_key_middleware():
    c = client(FakeEngine(), api_key="k")
    assert c.post("/v1/completions", json={"prompt": "x"}).status_code == 401
    ok = c.post("/v1/completions", json={"prompt": "x"}, headers={"Authorization": "Bearer k"})
    assert ok.status_code == 200
    assert c.get("/health").status_code == 200


def test_sampling_fields_reach_engine():
    e = FakeEngine()
    client(e).post("/v1/chat/completions", json={
        "messages": [{"role": "user", "content": "x"}], "temperature": 0.7, "top_p": 0.9, "top_k": 20,
        "min_p": 0.05, "presence_penalty": 0.5, "frequency_penalty": 0.2, "repetition_penalty": 1.1,
        "priority": 2, "stop_token_ids": [7], "response_format": {"type": "json_schema",
                                                                  "json_schema": {"schema": {"type": "object"}}}})
    sp = e.last_sp
    assert (sp.temperature, sp.top_p, sp.top_k, sp.min_p, sp.priority) == (0.7, 0.9, 20, 0.05, 2)
    assert sp.stop_token_ids == (7,) and sp.guided_json == {"type": "object"}


def test_cli_env_precedence(monkeypatch):
    monkeypatch.setenv("B200MOE_PORT", "9123")
    monkeypatch.setenv("NANOVLLM_MAX_NUM_SEQS", "33")
    a = build_parser().parse_args([])
    assert a.port == 9123 and a.max_num_seqs == 33
    a = build_parser().parse_args(["--port", "9000"])
    assert a.port == 9000
    assert is_loopback("127.0.0.1") and not is_loopback("0.0.0.0")
    with pytest.raises(SystemExit):
        main(["--model", "tiny-moe", "--host", "0.0.0.0"])


def test_real_async_engine_cpu_stream():
    eng = AsyncLLMEngine("tiny-moe", device="cpu", kvcache_block_size=16, num_kvcache_blocks=64,
                         max_num_batched_tokens=256, max_num_seqs=8, max_model_len=256, enforce_eager=True,
                         scheduler_policy="stall_free")
    try:
        c = TestClient(create_app(eng, "tiny"))
        r = c.post("/v1/completions", json={"prompt": list(range(20)), "max_tokens": 6, "temperature": 0,
                                             "stream": True})
        lines = [l for l in r.text.split("\n\n") if l]
        assert lines[-1] == "data: [DONE]"
        r2 = c.post("/v1/completions", json={"prompt": list(range(20)), "max_tokens": 6, "temperature": 0})
        assert r2.json()["usage"]["completion_tokens"] == 6
        m = eng.metrics()
        assert m["requests_finished"] >= 2 and m["generated_tokens_total"] >= 12
        assert "b200moe_engine_steps_total" in c.get("/metrics").text
        # admission: a prompt that exceeds max_model_len -> 400; KV capacity -> 429
        assert c.post("/v1/completions", json={"prompt": [1] * 300, "max_tokens": 4}).status_code == 400
    finally:
        asyncio.run(eng.close())


def test_client_disconnect_cancels_stream():
    """A streaming client that goes away: the request is cancelled in the
    engine (its KV blocks freed) instead of decoding to max_tokens
    (reference: nanovllm/entrypoints/api_server.py:224-226)."""

    class Endless(FakeEngine):
        async def add_request(self, prompt, sp):
            self._id += 1
            return RequestHandle(self._id, None)

        async def next_event(self, h):
            await asyncio.sleep(0.002)
            return TokenEvent(token_id=104, finished=False)

    eng = Endless()
    app = create_app(eng, "tiny")
    body = json.dumps({"model": "tiny", "prompt": "hi", "max_tokens": 100000, "stream": True}).encode()
    sent = []

    async def run():
        calls = {"n": 0}

        async def receive():
            calls["n"] += 1
            if calls["n"] == 1:
                return {"type": "http.request", "body": body, "more_body": False}
            await asyncio.sleep(0.05)  # the client reads a few chunks, then disconnects
            return {"type": "http.disconnect"}

        async def send(msg):
            sent.append(msg)

        scope = {"type": "http", "asgi": {"version": "3.0"}, "http_version": "1.1", "method": "POST",
                 "scheme": "http", "path": "/v1/completions", "raw_path": b"/v1/completions", "query_string": b"",
                 "headers": [(b"content-type", b"application/json"), (b"host", b"test")],
                 "client": ("127.0.0.1", 1), "server": ("127.0.0.1", 80), "root_path": ""}
        await asyncio.wait_for(app(scope, receive, send), 10)

    asyncio.run(run())
    assert eng.cancelled == [1]
    chunks = [m for m in sent if m["type"] == "http.response.body" and m.get("body")]
    assert 0 < len(chunks) < 1000
    assert not any(b"[DONE]" in m["body"] for m in chunks)


def test_cli_reference_flags(monkeypatch, capsys):
    """The reference server's remaining flags: backends and expert placement
    reach the engine, --allow-insecure permits a non-loopback bind without a
    key, --log-level reaches uvicorn, --version prints the version."""
    import uvicorn

    import b200moe
    import b200moe.async_engine as ae
    from b200moe.entrypoints.openai.api_server import engine_kwargs
    a = build_parser().parse_args(["--attention-backend", "triton_paged", "--decode-moe-backend", "grouped_mm",
                                   "--expert-placement", "round_robin", "--expert-map-path", "/x.json"])
    kw = engine_kwargs(a)
    assert (kw["attention_backend"], kw["decode_moe_backend"], kw["expert_placement"], kw["expert_map_path"]) == \
        ("triton_paged", "grouped_mm", "round_robin", "/x.json")
    assert engine_kwargs(build_parser().parse_args([]))["decode_moe_backend"] is None
    seen = {}
    monkeypatch.setattr(ae, "AsyncLLMEngine", lambda model, **kw: seen.update(kw=kw) or FakeEngine())
    monkeypatch.setattr(uvicorn, "run", lambda app, **kw: seen.update(run=kw))
    main(["--model", "tiny-moe", "--host", "0.0.0.0", "--allow-insecure", "--log-level", "warning"])
    assert seen["run"]["host"] == "0.0.0.0" and seen["run"]["log_level"] == "warning"
    with pytest.raises(SystemExit):
        build_parser().parse_args(["--version"])
    assert b200moe.__version__ in capsys.readouterr().out


def test_async_engine_many_streams_one_loop_queue_limit_and_cancel():
    """Real engine on CPU: eight concurrent streams on one event loop each get their
    tokens in order; with the queue at its limit a further request is refused
    (OverflowError) and counted; a cancelled stream ends with a cancelled event and
    its slot is free again."""
    from b200moe.sampling_params import SamplingParams
    eng = AsyncLLMEngine("tiny-moe", device="cpu", kvcache_block_size=16, num_kvcache_blocks=128,
                         max_num_batched_tokens=512, max_num_seqs=8, max_model_len=256, enforce_eager=True,
                         max_queue_size=8)
    sp = SamplingParams(temperature=0.0, max_tokens=5, ignore_eos=True)

    async def drain(h):
        toks = []
        while True:
            ev = await eng.next_event(h)
            assert ev.error is None
            if ev.token_id is not None:
                toks.append(ev.token_id)
            if ev.finished:
                return toks, ev

    async def run():
        handles = [await eng.add_request(list(range(3 + i, 20 + i)), sp) for i in range(8)]
        with pytest.raises(OverflowError):
            await eng.add_request([1, 2, 3], sp)
        results = await asyncio.gather(*(drain(h) for h in handles))
        assert all(len(t) == 5 and ev.metrics["output_tokens"] == 5 for t, ev in results)
        long_sp = SamplingParams(temperature=0.0, max_tokens=200, ignore_eos=True)
        h = await eng.add_request(list(range(10)), long_sp)
        first = await eng.next_event(h)
        assert first.token_id is not None
        eng.cancel(h.seq_id)
        while True:
            ev = await eng.next_event(h)
            if ev.finished:
                break
        assert ev.cancelled
        toks, _ = await drain(await eng.add_request([7, 8, 9], sp))  # the slot is usable again
        assert len(toks) == 5

    try:
        asyncio.run(run())
        m = eng.metrics()
        assert m["requests_rejected"] == 1 and m["requests_cancelled"] == 1
        assert m["requests_finished"] == 9 and m["active_requests"] == 0
    finally:
        asyncio.run(eng.close())
