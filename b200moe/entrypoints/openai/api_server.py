"""OpenAI-compatible HTTP server (reference: nanovllm/entrypoints/openai/api_server.py).

Routes: ``GET /health``, ``GET /v1/models``, ``GET /metrics`` (Prometheus text),
``POST /v1/chat/completions`` and ``POST /v1/completions``, both with SSE
streaming.  Request fields: max_tokens, temperature, top_p, top_k, min_p,
presence/frequency/repetition penalties, stop (strings, with retraction of the
matched text), stop_token_ids, logprobs (chat: bool + top_logprobs;
completions: int), response_format json_schema / guided_json / guided_regex,
priority, ignore_eos (decode to max_tokens), stream,
stream_options.include_usage / include_metrics.
Errors: 400 invalid request, 401 bad API key, 429 queue full / KV capacity,
500 engine error.  A client disconnect cancels the request.

CLI flags mirror the reference's and default from ``B200MOE_*`` (or the
reference's ``NANOVLLM_*``) environment variables; the command line wins.  The
server refuses to bind a non-loopback address without an API key.
"""
from __future__ import annotations

import argparse
import json
import os
import time
import uuid

from fastapi import FastAPI, Request
from fastapi.responses import JSONResponse, PlainTextResponse, StreamingResponse

from b200moe import __version__
from b200moe.incremental_detokenizer import IncrementalDetokenizer
from b200moe.sampling_params import SamplingParams

METRIC_KEYS = ("prompt_tokens", "output_tokens", "queue_s", "ttft_s", "e2e_s", "tpot_s", "mean_tpot_s",
               "itls_s", "finish_reason")


class BadRequest(Exception):
    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status
        self.message = message


def parse_sampling(body: dict, chat: bool) -> tuple[SamplingParams, list[str], dict]:
    """OpenAI request body -> (SamplingParams, stop strings, stream options)."""
    if body.get("n", 1) != 1:
        raise BadRequest(400, "only n=1 is supported")
    banned = ("tools", "tool_choice") if chat else ("tools", "tool_choice", "echo", "suffix", "best_of")
    bad = [k for k in banned if body.get(k) not in (None, False)]
    if bad:
        raise BadRequest(400, f"unsupported parameters: {', '.join(bad)}")

    def num(key, cast, default):
        try:
            return cast(body.get(key, default))
        except (TypeError, ValueError):
            raise BadRequest(400, f"{key} must be a number")

    max_tokens = num("max_tokens", int, 64)
    temperature = num("temperature", float, 1.0)
    priority = num("priority", int, 0)
    if max_tokens <= 0 or temperature < 0 or priority < 0:
        raise BadRequest(400, "max_tokens must be positive; temperature/priority non-negative")
    kw = dict(top_p=num("top_p", float, 1.0), top_k=num("top_k", int, -1), min_p=num("min_p", float, 0.0),
              presence_penalty=num("presence_penalty", float, 0.0),
              frequency_penalty=num("frequency_penalty", float, 0.0),
              repetition_penalty=num("repetition_penalty", float, 1.0),
              skip_special_tokens=bool(body.get("skip_special_tokens", True)),
              ignore_eos=bool(body.get("ignore_eos", False)))
    if body.get("seed") is not None:
        kw["seed"] = num("seed", int, 0)
    stop_ids = body.get("stop_token_ids")
    if stop_ids is not None:
        if not isinstance(stop_ids, list) or not all(isinstance(t, int) and not isinstance(t, bool) for t in stop_ids):
            raise BadRequest(400, "stop_token_ids must be a list of integers")
        kw["stop_token_ids"] = stop_ids
    if chat:
        if body.get("logprobs"):
            kw["logprobs"] = max(1, num("top_logprobs", int, 0))
    elif body.get("logprobs") is not None:
        kw["logprobs"] = num("logprobs", int, 0)
    rf = body.get("response_format")
    if rf is not None:
        if not isinstance(rf, dict) or rf.get("type") != "json_schema":
            raise BadRequest(400, "response_format.type must be 'json_schema'")
        js = rf.get("json_schema")
        schema = js.get("schema") if isinstance(js, dict) else None
        if schema is None and isinstance(js, dict) and js:
            schema = js
        if not isinstance(schema, (dict, str)):
            raise BadRequest(400, "response_format.json_schema.schema must be an object")
        kw["guided_json"] = schema
    if body.get("guided_json") is not None:
        kw["guided_json"] = body["guided_json"]
    if body.get("guided_regex") is not None:
        kw["guided_regex"] = body["guided_regex"]
    stop = body.get("stop", [])
    if isinstance(stop, str):
        stop = [stop]
    if not isinstance(stop, list) or not all(isinstance(s, str) for s in stop):
        raise BadRequest(400, "stop must be a string or list of strings")
    opts = body.get("stream_options") or {}
    if not isinstance(opts, dict):
        raise BadRequest(400, "stream_options must be an object")
    try:
        sp = SamplingParams(temperature=temperature, max_tokens=max_tokens, priority=priority, **kw)
    except (ValueError, AssertionError) as exc:
        raise BadRequest(400, str(exc))
    return sp, stop, opts


class _Stream:
    """Accumulates decoded text for one request and applies stop strings."""

    def __init__(self, tokenizer, sp: SamplingParams, stop: list[str]):
        self.tok = tokenizer
        self.decoder = IncrementalDetokenizer(tokenizer, skip_special_tokens=sp.skip_special_tokens)
        self.stop = stop
        self.text = ""
        self.token_ids: list[int] = []
        self.stopped = False

    def push(self, token_id: int) -> str:
        self.token_ids.append(token_id)
        delta = self.decoder.push(token_id)
        self.text += delta
        hit = next((s for s in self.stop if s in self.text), None)
        if hit is not None:
            visible = self.text.split(hit, 1)[0]
            cut = len(self.text) - len(visible)
            delta = delta[:-cut] if 0 < cut <= len(delta) else ("" if cut else delta)
            self.text = visible
            self.stopped = True
        return delta


def create_app(engine, model_name: str, api_key: str | None = None, version: str | None = __version__):
    app = FastAPI(title="b200moe")
    tokenizer = engine.tokenizer
    tok_cache: dict[int, str] = {}

    def tstr(t: int) -> str:
        s = tok_cache.get(t)
        if s is None:
            s = tok_cache[t] = tokenizer.decode([t])
        return s

    def err(status, message, kind="invalid_request_error"):
        return JSONResponse(status_code=status, content={"error": {"message": message, "type": kind}})

    if api_key:
        @app.middleware("http")
        async def auth(request: Request, call_next):
            if request.url.path.startswith("/v1/") and request.headers.get("authorization") != f"Bearer {api_key}":
                return err(401, "invalid API key")
            return await call_next(request)

    @app.exception_handler(BadRequest)
    async def _bad(request, exc: BadRequest):
        return err(exc.status, exc.message, "engine_error" if exc.status >= 500 else "invalid_request_error")

    @app.on_event("shutdown")
    async def _shutdown():
        await engine.close()

    @app.get("/health")
    async def health():
        d = {"status": "ok", "model": model_name}
        if version:
            d["version"] = version
        return d

    @app.get("/v1/models")
    async def models():
        return {"object": "list", "data": [{"id": model_name, "object": "model", "owned_by": "local"}]}

    @app.get("/metrics")
    async def metrics():
        return PlainTextResponse(engine.prometheus_text())

    async def submit(prompt_ids, sp):
        try:
            return await engine.add_request(prompt_ids, sp)
        except OverflowError as exc:
            raise BadRequest(429, str(exc))
        except ValueError as exc:
            raise BadRequest(400, str(exc))

    def chat_lp(token_id, lp):
        t = tstr(token_id)
        return {"token": t, "logprob": lp["chosen"], "bytes": list(t.encode()),
                "top_logprobs": [{"token": tstr(i), "logprob": v, "bytes": list(tstr(i).encode())}
                                 for i, v in lp["top"]]}

    def completion_lp(entries, offsets):
        return {"tokens": [tstr(t) for t, _ in entries], "token_logprobs": [lp["chosen"] for _, lp in entries],
                "top_logprobs": [{tstr(i): v for i, v in lp["top"]} for _, lp in entries],
                "text_offset": offsets}

    async def run(request: Request, prompt_ids, sp, stop, opts, chat: bool):
        handle = await submit(prompt_ids, sp)
        rid = f"{'chatcmpl' if chat else 'cmpl'}-{uuid.uuid4().hex}"
        created = int(time.time())
        obj = "chat.completion" if chat else "text_completion"
        st = _Stream(tokenizer, sp, stop)
        usage = lambda: {"prompt_tokens": len(prompt_ids), "completion_tokens": len(st.token_ids),
                         "total_tokens": len(prompt_ids) + len(st.token_ids)}

        def choice(delta_text, finish, lp=None):
            if chat:
                c = {"index": 0, "delta": {"content": delta_text} if delta_text is not None else {},
                     "finish_reason": finish}
            else:
                c = {"index": 0, "text": delta_text or "", "finish_reason": finish, "logprobs": None}
            if lp is not None:
                c["logprobs"] = lp
            return c

        def chunk(choices, **extra):
            d = {"id": rid, "object": obj + ".chunk" if chat else obj, "created": created, "model": model_name,
                 "choices": choices}
            d.update(extra)
            return f"data: {json.dumps(d, ensure_ascii=False)}\n\n"

        async def events():
            finish = "length"
            offset = 0
            try:
                while True:
                    if await request.is_disconnected():
                        engine.cancel(handle.seq_id)
                        return
                    ev = await engine.next_event(handle)
                    if ev.error:
                        yield f"data: {json.dumps({'error': {'message': ev.error, 'type': 'engine_error'}})}\n\n"
                        return
                    if ev.cancelled:
                        return
                    if ev.token_id is not None:
                        delta = st.push(ev.token_id)
                        lp = None
                        if ev.logprobs is not None:
                            lp = ({"content": [chat_lp(ev.token_id, ev.logprobs)]} if chat
                                  else completion_lp([(ev.token_id, ev.logprobs)], [offset]))
                        offset += len(delta)
                        if delta or lp is not None:
                            yield chunk([choice(delta, None, lp)])
                        if st.stopped:
                            engine.cancel(handle.seq_id)
                            finish = "stop"
                            ev.finished = True
                    if ev.finished:
                        if ev.metrics and ev.metrics.get("finish_reason") and not st.stopped:
                            finish = ev.metrics["finish_reason"]
                        extra = {}
                        if opts.get("include_metrics") and ev.metrics:
                            extra["metrics"] = {k: ev.metrics[k] for k in METRIC_KEYS if k in ev.metrics}
                        yield chunk([choice(None if chat else "", finish)], **extra)
                        if opts.get("include_usage"):
                            yield chunk([], usage=usage())
                        yield "data: [DONE]\n\n"
                        return
            finally:
                engine.cancel(handle.seq_id)

        if request.state.stream:
            return StreamingResponse(events(), media_type="text/event-stream")
        finish, lps, offsets = "length", [], []
        try:
            while True:
                ev = await engine.next_event(handle)
                if ev.error:
                    raise BadRequest(500, ev.error)
                if ev.cancelled:
                    break
                if ev.token_id is not None:
                    offsets.append(len(st.text))
                    st.push(ev.token_id)
                    if ev.logprobs is not None:
                        lps.append((ev.token_id, ev.logprobs))
                    if st.stopped:
                        finish = "stop"
                        break
                if ev.finished:
                    if ev.metrics and ev.metrics.get("finish_reason"):
                        finish = ev.metrics["finish_reason"]
                    break
        finally:
            engine.cancel(handle.seq_id)
        if chat:
            c = {"index": 0, "message": {"role": "assistant", "content": st.text}, "finish_reason": finish,
                 "logprobs": {"content": [chat_lp(t, lp) for t, lp in lps]} if lps else None}
        else:
            c = {"index": 0, "text": st.text, "finish_reason": finish,
                 "logprobs": completion_lp(lps, offsets[:len(lps)]) if lps else None}
        return JSONResponse({"id": rid, "object": obj, "created": created, "model": model_name, "choices": [c],
                             "usage": usage()})

    @app.post("/v1/chat/completions")
    async def chat_completions(request: Request):
        try:
            body = await request.json()
        except Exception:
            raise BadRequest(400, "request body must be JSON")
        sp, stop, opts = parse_sampling(body, chat=True)
        msgs = body.get("messages")
        if not isinstance(msgs, list) or not msgs:
            raise BadRequest(400, "messages must be a non-empty list")
        try:
            ids = tokenizer.apply_chat_template(msgs, tokenize=True, add_generation_prompt=True)
        except Exception as exc:
            raise BadRequest(400, f"invalid chat messages: {exc}")
        if hasattr(ids, "keys"):
            ids = ids["input_ids"]
        if hasattr(ids, "tolist"):
            ids = ids.tolist()
        if ids and isinstance(ids[0], (list, tuple)):
            ids = ids[0]
        ids = [int(t) for t in ids]
        if not ids:
            raise BadRequest(400, "chat template produced an empty prompt")
        request.state.stream = bool(body.get("stream", False))
        return await run(request, ids, sp, stop, opts, chat=True)

    @app.post("/v1/completions")
    async def completions(request: Request):
        try:
            body = await request.json()
        except Exception:
            raise BadRequest(400, "request body must be JSON")
        sp, stop, opts = parse_sampling(body, chat=False)
        prompt = body.get("prompt")
        if isinstance(prompt, str):
            ids = tokenizer.encode(prompt)
        elif isinstance(prompt, list) and prompt and all(isinstance(t, int) and not isinstance(t, bool) for t in prompt):
            ids = [int(t) for t in prompt]
        else:
            raise BadRequest(400, "prompt must be a string or a list of token ids")
        if not ids:
            raise BadRequest(400, "prompt produced an empty token list")
        request.state.stream = bool(body.get("stream", False))
        return await run(request, ids, sp, stop, opts, chat=False)

    return app


# ----------------------------------------------------------------------- CLI
def _env(name: str, default=None):
    return os.environ.get(f"B200MOE_{name}", os.environ.get(f"NANOVLLM_{name}", default))


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="b200moe OpenAI-compatible server")
    p.add_argument("--model", default=_env("MODEL"))
    p.add_argument("--served-model-name", default=_env("SERVED_MODEL_NAME"))
    p.add_argument("--host", default=_env("HOST", "127.0.0.1"))
    p.add_argument("--port", type=int, default=int(_env("PORT", "8000")))
    p.add_argument("--api-key", default=_env("API_KEY"))
    p.add_argument("--tensor-parallel-size", type=int, default=int(_env("TENSOR_PARALLEL_SIZE", "1")))
    p.add_argument("--expert-parallel-size", type=int, default=int(_env("EXPERT_PARALLEL_SIZE", "0")))
    p.add_argument("--attention-parallel", default=_env("ATTENTION_PARALLEL", "dp"), choices=["dp", "tp"])
    p.add_argument("--moe-backend", default=_env("MOE_BACKEND", "fused"))
    p.add_argument("--max-model-len", type=int, default=int(_env("MAX_MODEL_LEN", "4096")))
    p.add_argument("--max-num-seqs", type=int, default=int(_env("MAX_NUM_SEQS", "256")))
    p.add_argument("--max-num-batched-tokens", type=int, default=int(_env("MAX_NUM_BATCHED_TOKENS", "16384")))
    p.add_argument("--gpu-memory-utilization", type=float, default=float(_env("GPU_MEMORY_UTILIZATION", "0.9")))
    p.add_argument("--kvcache-block-size", type=int, default=int(_env("KVCACHE_BLOCK_SIZE", "256")))
    p.add_argument("--kv-cache-dtype", default=_env("KV_CACHE_DTYPE", "bf16"), choices=["bf16", "int8"])
    p.add_argument("--kv-int8-mode", default=_env("KV_INT8_MODE", "token"), choices=["token", "channel"],
                   help="int8 KV: per token-head scales, or the reference's calibrated per-channel scales")
    p.add_argument("--scheduler-policy", default=_env("SCHEDULER_POLICY", "stall_free"),
                   choices=["fcfs", "stall_free", "stall_free_lpm"])
    p.add_argument("--prefill-chunk-size", type=int, default=int(_env("PREFILL_CHUNK_SIZE", "256")))
    p.add_argument("--scheduler-overlap", action="store_true", default=_env("SCHEDULER_OVERLAP", "0") == "1")
    p.add_argument("--kv-offload", action="store_true", default=_env("KV_OFFLOAD", "0") == "1")
    p.add_argument("--kv-offload-host-blocks", type=int, default=int(_env("KV_OFFLOAD_HOST_BLOCKS", "256")))
    p.add_argument("--enforce-eager", action="store_true", default=_env("ENFORCE_EAGER", "0") == "1")
    p.add_argument("--max-queue-size", type=int, default=int(_env("MAX_QUEUE_SIZE", "1024")))
    p.add_argument("--random-init", action="store_true", default=_env("RANDOM_INIT", "0") == "1",
                   help="random weights of the checkpoint's architecture (no weight files needed)")
    p.add_argument("--metrics-path", default=_env("METRICS_PATH"))
    p.add_argument("--device", default=_env("DEVICE", "cuda"), choices=["cuda", "cpu"])
    p.add_argument("--attention-backend", default=_env("ATTENTION_BACKEND", "paged"))
    p.add_argument("--decode-moe-backend", default=_env("DECODE_MOE_BACKEND"))
    p.add_argument("--expert-placement", default=_env("EXPERT_PLACEMENT", "linear"),
                   choices=["linear", "round_robin", "profiled"])
    p.add_argument("--expert-map-path", default=_env("EXPERT_MAP_PATH"))
    p.add_argument("--allow-insecure", action="store_true", default=_env("ALLOW_INSECURE", "0") == "1",
                   help="allow a non-loopback bind without an API key (trusted networks only)")
    p.add_argument("--log-level", default=_env("LOG_LEVEL", "info"),
                   choices=["critical", "error", "warning", "info", "debug", "trace"])
    from b200moe import __version__
    p.add_argument("--version", action="version", version=f"%(prog)s {__version__}")
    return p


def engine_kwargs(a) -> dict:
    return dict(tensor_parallel_size=a.tensor_parallel_size, expert_parallel_size=a.expert_parallel_size,
                attention_parallel=a.attention_parallel, moe_backend=a.moe_backend, max_model_len=a.max_model_len,
                max_num_seqs=a.max_num_seqs, max_num_batched_tokens=a.max_num_batched_tokens,
                gpu_memory_utilization=a.gpu_memory_utilization, kvcache_block_size=a.kvcache_block_size,
                kv_cache_dtype=a.kv_cache_dtype, kv_int8_mode=a.kv_int8_mode, scheduler_policy=a.scheduler_policy,
                prefill_chunk_size=a.prefill_chunk_size, scheduler_overlap=a.scheduler_overlap,
                kv_offload_enabled=a.kv_offload, kv_offload_host_blocks=a.kv_offload_host_blocks,
                enforce_eager=a.enforce_eager, max_queue_size=a.max_queue_size, metrics_path=a.metrics_path,
                random_init="seeded" if a.random_init else "", device=a.device,
                attention_backend=a.attention_backend, decode_moe_backend=a.decode_moe_backend or None,
                expert_placement=a.expert_placement, expert_map_path=a.expert_map_path or None)


def is_loopback(host: str) -> bool:
    return host in ("127.0.0.1", "localhost", "::1") or host.startswith("127.")


def main(argv=None):
    a = build_parser().parse_args(argv)
    if not a.model:
        raise SystemExit("--model (or B200MOE_MODEL) is required")
    if not is_loopback(a.host) and not a.api_key and not a.allow_insecure:
        raise SystemExit(f"refusing to bind {a.host} without --api-key (or --allow-insecure on a trusted network)")
    import uvicorn
    from b200moe.async_engine import AsyncLLMEngine
    engine = AsyncLLMEngine(a.model, **engine_kwargs(a))
    app = create_app(engine, a.served_model_name or os.path.basename(a.model.rstrip("/")), a.api_key)
    uvicorn.run(app, host=a.host, port=a.port, log_level=a.log_level)


if __name__ == "__main__":
    main()
