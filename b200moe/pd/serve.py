"""Prefill / decode disaggregated serving roles (plus the collocated arm).

    python -m b200moe.pd.serve --role decode    --model M --port 9100 [--kv-transport nvlink]
    python -m b200moe.pd.serve --role prefill   --model M --port 9000 --d-port 9100
    python -m b200moe.pd.serve --role collocated --model M --port 9000

Client protocol (framed JSON, ``b200moe.pd.protocol``) on ``--port`` of the
prefill or collocated role: requests ``{"req_id", "prompt" (ids or text),
"max_tokens", "priority"?}``, a final ``{"type": "done"}``; replies
``{"type": "result", "req_id", "tokens", "metrics", "prefill_s"?}``.

Prefill <-> decode: the decode role listens on ``--port`` (KV frames, TCP
transport) and ``--port + 1`` (control).  A finished prefill (prompt computed,
first token sampled) is handed off:

* ``tcp``     prefill sends ``handoff`` (token ids, sampling, block count) and
              then the KV frame; decode reserves blocks (back-pressure while
              its pool is full), imports the frame, starts decoding.
* ``nvlink``  decode first publishes its pool's CUDA IPC handle (``pool``);
              on ``handoff`` it reserves blocks and answers ``blocks``; prefill
              copies the slabs into them over NVLink and sends ``kv_ready``.

The prefill engine then releases the sequence; the decode engine returns
``result`` messages, which prefill forwards to its client.  Behaviour
follows the reference's roles (scripts/p15_pd_serve.py:55-296).
"""
from __future__ import annotations

import argparse
import selectors
import time
from collections import deque

from b200moe.pd.kv_channel import KVFrameAssembler, NvlinkKVChannel, TcpKVChannel, export_pool_handle
from b200moe.pd.protocol import JsonStream, connect_retry, listen, send_json


def build_engine(args, **extra):
    from b200moe.engine.llm_engine import LLMEngine
    kw = dict(max_num_seqs=args.max_num_seqs, max_model_len=args.max_model_len, scheduler_overlap=False,
              kvcache_block_size=args.kvcache_block_size, enforce_eager=args.enforce_eager,
              max_num_batched_tokens=args.max_num_batched_tokens, scheduler_policy=args.scheduler_policy)
    if args.num_kvcache_blocks:
        kw["num_kvcache_blocks"] = args.num_kvcache_blocks
    if args.random_init:
        kw["random_init"] = "seeded"
    if args.device:
        kw["device"] = args.device
    kw.update(extra)
    return LLMEngine(args.model, **kw)


def sampling_params(msg: dict):
    from b200moe import SamplingParams
    return SamplingParams(temperature=float(msg.get("temperature", 0.0)), max_tokens=int(msg["max_tokens"]),
                          ignore_eos=bool(msg.get("ignore_eos", True)), priority=int(msg.get("priority", 0)))


def _read(sel, streams: dict):
    """Poll the sockets once: yields (socket, [messages or raw frames]); None on EOF."""
    for key, _ in sel.select(timeout=0.02):
        sock = key.fileobj
        try:
            chunk = sock.recv(1 << 22)
        except BlockingIOError:
            continue
        if not chunk:
            yield sock, None
            continue
        yield sock, streams[sock].feed(chunk)


def _live(engine) -> bool:
    return not engine.is_finished()


# ------------------------------------------------------------------ collocated
def role_collocated(args):
    eng = build_engine(args, tensor_parallel_size=args.tensor_parallel_size)
    srv = listen(args.port)
    print(f"[collocated] listening on {args.port}", flush=True)
    client, _ = srv.accept()
    client.setblocking(False)
    sel = selectors.DefaultSelector()
    sel.register(client, selectors.EVENT_READ)
    streams = {client: JsonStream()}
    req = {}
    running = True
    while running or _live(eng):
        for sock, msgs in _read(sel, streams):
            if msgs is None:
                running = False
                break
            for m in msgs:
                if m.get("type") == "done":
                    running = False
                else:
                    req[eng.add_request(m["prompt"], sampling_params(m))] = m["req_id"]
        if _live(eng):
            outputs, _ = eng.step()
            for sid, toks, metrics in outputs:
                send_json(client, {"type": "result", "req_id": req.pop(sid), "tokens": list(toks),
                                   "metrics": metrics})
        elif not running:
            break
    client.close()
    eng.exit()
    print("[collocated] clean exit", flush=True)


# ------------------------------------------------------------------ decode
def role_decode(args):
    eng = build_engine(args)
    pool = eng.executor.runner.kv
    kv_srv, ctrl_srv = listen(args.port), listen(args.port + 1)
    print(f"[decode] listening on {args.port}/{args.port + 1} ({args.kv_transport})", flush=True)
    kv_sock, _ = kv_srv.accept()
    ctrl, _ = ctrl_srv.accept()
    for s in (kv_sock, ctrl):
        s.setblocking(False)
    tcp = TcpKVChannel(kv_sock, pool, max_blocks=16)
    if args.kv_transport == "nvlink":
        send_json(ctrl, {"type": "pool", **export_pool_handle(pool)})
    sel = selectors.DefaultSelector()
    sel.register(kv_sock, selectors.EVENT_READ)
    sel.register(ctrl, selectors.EVENT_READ)
    streams = {kv_sock: KVFrameAssembler(), ctrl: JsonStream()}
    hold = deque()      # handoffs waiting for free blocks (back-pressure)
    pending = deque()   # (req_id, seq) with reserved blocks, waiting for their KV (tcp: FIFO)
    waiting_nv = {}     # req_id -> seq (nvlink: blocks sent, waiting for kv_ready)
    frames = deque()
    fin = {}
    running = True
    while running or _live(eng) or pending or waiting_nv:
        for sock, msgs in _read(sel, streams):
            if msgs is None:
                running = False
                break
            if sock is kv_sock:
                frames.extend(msgs)
                continue
            for m in msgs:
                t = m.get("type")
                if t == "done":
                    running = False
                elif t == "handoff":
                    hold.append(m)
                elif t == "kv_ready":
                    seq = waiting_nv.pop(m["req_id"])
                    eng.activate(seq)
                    fin[seq.seq_id] = m["req_id"]
        while hold:
            m = hold[0]
            seq = eng.admit_prefilled(m["token_ids"], m["num_prompt_tokens"], sampling_params(m))
            if seq is None:
                break
            hold.popleft()
            if args.kv_transport == "nvlink":
                waiting_nv[m["req_id"]] = seq
                send_json(ctrl, {"type": "blocks", "req_id": m["req_id"], "block_ids": seq.block_table})
            else:
                pending.append((m["req_id"], seq))
        while pending and frames:
            rid, seq = pending.popleft()
            tcp.import_frame(seq.block_table, frames.popleft())
            eng.activate(seq)
            fin[seq.seq_id] = rid
        if _live(eng):
            outputs, _ = eng.step()
            for sid, toks, metrics in outputs:
                send_json(ctrl, {"type": "result", "req_id": fin.pop(sid), "tokens": list(toks), "metrics": metrics})
        elif not running and not pending and not waiting_nv:
            break
    kv_sock.close()
    ctrl.close()
    eng.exit()
    print("[decode] clean exit", flush=True)


# ------------------------------------------------------------------ prefill
def role_prefill(args):
    eng = build_engine(args)
    pool = eng.executor.runner.kv
    kv_sock = connect_retry(args.host, args.d_port)
    ctrl = connect_retry(args.host, args.d_port + 1)
    tcp = TcpKVChannel(kv_sock, pool, max_blocks=16)
    nv = None
    srv = listen(args.port)
    print(f"[prefill] client port {args.port}, decode at {args.d_port} ({args.kv_transport})", flush=True)
    client, _ = srv.accept()
    client.setblocking(False)
    sel = selectors.DefaultSelector()
    sel.register(client, selectors.EVENT_READ)
    sel.register(ctrl, selectors.EVENT_READ)
    streams = {client: JsonStream(), ctrl: JsonStream()}
    t_add, rid_of, handed, prefill_s, sent = {}, {}, {}, {}, set()
    outstanding = 0
    running = True
    while running or _live(eng) or outstanding:
        for sock, msgs in _read(sel, streams):
            if msgs is None:
                running = False
                outstanding = 0
                break
            for m in msgs:
                t = m.get("type")
                if sock is client:
                    if t == "done":
                        running = False
                        continue
                    sid = eng.add_request(m["prompt"], sampling_params(m))
                    t_add[sid], rid_of[sid] = time.perf_counter(), m["req_id"]
                    outstanding += 1
                elif t == "pool":
                    nv = NvlinkKVChannel(pool, m)
                elif t == "blocks":  # nvlink: the decode side reserved these blocks
                    seq, nblocks = handed.pop(m["req_id"])
                    nv.send_blocks(seq.block_table[:nblocks], m["block_ids"][:nblocks])
                    send_json(ctrl, {"type": "kv_ready", "req_id": m["req_id"]})
                    eng.release(seq)
                elif t == "result":
                    outstanding -= 1
                    send_json(client, {**m, "prefill_s": prefill_s.get(m["req_id"])})
        if _live(eng):
            eng.step()
        for seq in eng.prefilled_sequences():
            if seq.seq_id in sent or seq.seq_id not in rid_of:
                continue
            rid = rid_of[seq.seq_id]
            sent.add(seq.seq_id)
            prefill_s[rid] = time.perf_counter() - t_add[seq.seq_id]
            nblocks = -(-(seq.num_tokens - 1) // eng.config.kvcache_block_size)  # blocks holding computed KV
            send_json(ctrl, {"type": "handoff", "req_id": rid, "token_ids": list(seq.tokens),
                             "num_prompt_tokens": seq.prompt_len, "max_tokens": seq.params.max_tokens,
                             "temperature": seq.params.temperature, "ignore_eos": seq.params.ignore_eos,
                             "priority": seq.params.priority, "nblocks": nblocks})
            if args.kv_transport == "nvlink":
                handed[rid] = (seq, nblocks)  # blocks stay allocated until the copy ("blocks")
                eng.detach(seq)
            else:
                tcp.send_blocks(seq.block_table[:nblocks])
                eng.cancel_request(seq.seq_id)
        if not running and not _live(eng) and outstanding <= 0:
            break
    send_json(ctrl, {"type": "done"})
    if nv is not None:
        nv.close()
    client.close()
    eng.exit()
    print("[prefill] clean exit", flush=True)


# ------------------------------------------------------------------ client
def run_client(host: str, port: int, requests: list[dict], timeout_s: float = 300.0) -> dict:
    """Send requests, then ``done``; returns {req_id: result message}."""
    sock = connect_retry(host, port, blocking=True)
    for r in requests:
        send_json(sock, r)
    js, results = JsonStream(), {}
    sock.settimeout(timeout_s)
    while len(results) < len(requests):
        chunk = sock.recv(1 << 20)
        if not chunk:
            break
        for m in js.feed(chunk):
            if m.get("type") == "result":
                results[m["req_id"]] = m
    send_json(sock, {"type": "done"})
    sock.close()
    return results


def parse_args(argv=None):
    p = argparse.ArgumentParser(description="PD disaggregated serving roles")
    p.add_argument("--role", required=True, choices=("collocated", "prefill", "decode"))
    p.add_argument("--model", required=True)
    p.add_argument("--random-init", action="store_true")
    p.add_argument("--device", default=None)
    p.add_argument("--port", type=int, default=9000)
    p.add_argument("--host", default="127.0.0.1", help="decode role's host (prefill connects to it)")
    p.add_argument("--d-port", type=int, default=9100, help="decode role's KV port; control is d-port + 1")
    p.add_argument("--kv-transport", choices=("tcp", "nvlink"), default="tcp")
    p.add_argument("--tensor-parallel-size", type=int, default=1, help="collocated role only")
    p.add_argument("--max-num-seqs", type=int, default=64)
    p.add_argument("--max-model-len", type=int, default=4096)
    p.add_argument("--max-num-batched-tokens", type=int, default=8192)
    p.add_argument("--kvcache-block-size", type=int, default=256)
    p.add_argument("--num-kvcache-blocks", type=int, default=0)
    p.add_argument("--scheduler-policy", default="fcfs")
    p.add_argument("--enforce-eager", action="store_true")
    return p.parse_args(argv)


def main(argv=None):
    a = parse_args(argv)
    {"collocated": role_collocated, "prefill": role_prefill, "decode": role_decode}[a.role](a)


if __name__ == "__main__":
    main()
