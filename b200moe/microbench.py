"""Kernel microbenchmarks on the 30B-A3B shapes, timed with CUDA events.

    python -m b200moe.microbench <case> [--tokens T] [--iters N]

cases:
  moe        grouped gate_up+SiLU and down GEMMs of one MoE layer (128 experts,
             T tokens x top-8, uniform random routing)
  dense      QKV (5120x2048) and O-proj (2048x4096) block-scaled GEMMs, LM head
  decode     paged decode attention, T sequences of --ctx tokens
  prefill    paged prefill attention, T/--ctx sequences of --ctx tokens
  step       whole-model forward (eager) of T decode rows at --ctx context
  ep         one expert-parallel MoE layer per rank under torchrun (fused peer-memory path)
  tp         tensor-parallel O projection + rank sum + RMSNorm under torchrun, fused vs NCCL
  all        every kernel case above

Each case prints a JSON line per kernel: milliseconds per call, the bytes or
FLOPs it must move, and the achieved fraction of the measured peaks (copy
bandwidth and cuBLAS bf16 throughput; MEASURED_PEAKS.json when present,
else 6.65 TB/s and 1.59 PFLOP/s).  Inputs are larger than L2 for the
bandwidth-bound cases, and a 256 MB buffer is rewritten between iterations.
"""
from __future__ import annotations

import argparse
import json
import math
import os

import torch

from b200moe import ops
from b200moe.utils.weights import quantize_block_fp8

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return d["hbm_gbs"] * 1e9, d["bf16_tflops"] * 1e12, "measured"
    except Exception:
        return 6.65e12, 1.59e15, "fallback"


_flush = None


def flush_l2():
    global _flush
    if _flush is None:
        _flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    _flush.fill_(1)


def _graph(fn, reps):
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.graph(g, stream=s):
        for _ in range(reps):
            fn()
    torch.cuda.synchronize()
    return g


# e4m3 weights in the tile-major layout the engine uses (B200MOE_TILED_WEIGHTS=0: row-major)
TILED = os.environ.get("B200MOE_TILED_WEIGHTS", "1") != "0"


def _time_graph(g, iters):
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    g.replay()
    torch.cuda.synchronize()
    a.record()
    for _ in range(iters):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


def timeit(fn, iters=20, warmup=3, flush=True, reps=10):
    """Device time of one call: ``reps`` calls (each after an L2 flush) are
    captured in a CUDA graph so host launch cost is excluded; the flush-only
    graph's time is subtracted."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if flush:
        flush_l2()
        work = _graph(lambda: (flush_l2(), fn()), reps)
        base = _graph(flush_l2, reps)
        return max(0.0, (_time_graph(work, iters) - _time_graph(base, iters)) / reps)
    return _time_graph(_graph(fn, reps), iters) / reps


def report(name, ms, bytes_=0, flops=0, **extra):
    bw, tf, src = peaks()
    d = {"kernel": name, "ms": round(ms, 4)}
    if bytes_:
        d["GB/s"] = round(bytes_ / ms / 1e6, 1)
        d["hbm_frac"] = round(bytes_ / (ms / 1e3) / bw, 3)
    if flops:
        d["TFLOP/s"] = round(flops / ms / 1e9, 1)
        d["tc_frac"] = round(flops / (ms / 1e3) / tf, 3)
    d["peak"] = src
    d.update(extra)
    print(json.dumps(d), flush=True)
    return d


def fp8_weight(groups, n, k, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    qs, ss = [], []
    for i in range(groups):
        q, s = quantize_block_fp8(torch.randn(n, k, generator=g, device="cuda") * 0.02)
        qs.append(q)
        ss.append(s)
    return torch.stack(qs), torch.stack(ss)


def case_moe(T, iters, E=128, k=8, H=2048, I=768, only=""):
    q13, s13 = fp8_weight(E, 2 * I, H, 1)
    q2, s2 = fp8_weight(E, H, I, 2)
    if TILED:
        q13, q2 = ops.tile_fp8(q13), ops.tile_fp8(q2)
    rows = T * k
    ids = torch.stack([torch.randperm(E, device="cuda")[:k] for _ in range(T)]).flatten()
    counts = torch.bincount(ids, minlength=E).to(torch.int32)
    offsets = torch.zeros(E + 1, dtype=torch.int32, device="cuda")
    offsets[1:] = torch.cumsum(counts, 0)
    x = (torch.randn(rows, H, device="cuda") * 0.5).to(torch.bfloat16)
    h = torch.empty(rows, I, dtype=torch.bfloat16, device="cuda")
    slots = torch.empty(rows, H, dtype=torch.bfloat16, device="cuda")
    sor = torch.randperm(rows, device="cuda").to(torch.int32)
    w = torch.rand(rows, device="cuda")
    used = int((counts > 0).sum())
    if only != "down":
        ms = timeit(lambda: ops.grouped_gate_up_silu(x, q13, s13, counts, offsets, h, I, tiled=TILED), iters)
        wbytes = used * 2 * I * H + rows * H * 2 + rows * I * 2
        report("moe_gate_up_silu", ms, wbytes, 2 * rows * H * 2 * I, tokens=T,
               bn=ops.pick_bn(rows, I // 128, E, pair=True))
    if rows >= 512 * E and only == "":
        # large prefill batch path: dequantise once, bf16 GEMMs (the dequantisation is timed)
        w13b = torch.empty(E, 2 * I, H, dtype=torch.bfloat16, device="cuda")
        w2b = torch.empty(E, H, I, dtype=torch.bfloat16, device="cuda")
        ms = timeit(lambda: (ops.dequant_weights(q13, s13, w13b, TILED),
                             ops.grouped_gate_up_silu(x, w13b, None, counts, offsets, h, I)), iters)
        report("moe_gate_up_silu_bf16once", ms, used * 2 * I * H * 3 + rows * H * 2 + rows * I * 2,
               2 * rows * H * 2 * I, tokens=T)
        ms = timeit(lambda: (ops.dequant_weights(q2, s2, w2b, TILED),
                             ops.grouped_down_scatter(h, w2b, None, counts, offsets, sor, w, slots)), iters)
        report("moe_down_scatter_bf16once", ms, used * H * I * 3 + rows * I * 2 + rows * H * 2,
               2 * rows * I * H, tokens=T)
    if only == "gate_up":
        return
    ms = timeit(lambda: ops.grouped_down_scatter(h, q2, s2, counts, offsets, sor, w, slots, tiled=TILED), iters)
    wbytes = used * H * I + rows * I * 2 + rows * H * 2
    report("moe_down_scatter", ms, wbytes, 2 * rows * I * H, tokens=T, bn=ops.pick_bn(rows, H // 128, E))


def case_dense(T, iters, H=2048):
    x = (torch.randn(T, H, device="cuda") * 0.5).to(torch.bfloat16)
    q, s = fp8_weight(1, 5120, H, 3)
    q = ops.tile_fp8(q) if TILED else q
    ms = timeit(lambda: ops.linear(x, q[0], s[0], tiled=TILED), iters)
    report("qkv_proj", ms, 5120 * H + T * (H + 5120) * 2, 2 * T * H * 5120, tokens=T)
    xo = (torch.randn(T, 4096, device="cuda") * 0.5).to(torch.bfloat16)
    q, s = fp8_weight(1, H, 4096, 4)
    q = ops.tile_fp8(q) if TILED else q
    ms = timeit(lambda: ops.linear(xo, q[0], s[0], tiled=TILED), iters)
    report("o_proj", ms, H * 4096 + T * (H + 4096) * 2, 2 * T * H * 4096, tokens=T)
    lm = (torch.randn(151936, H, device="cuda") * 0.02).to(torch.bfloat16)
    rows = min(T, 512)
    ms = timeit(lambda: ops.linear(x[:rows], lm, None, out_dtype=torch.float32), iters)
    report("lm_head", ms, 151936 * H * 2 + rows * 151936 * 4, 2 * rows * H * 151936, tokens=rows)


def _kv(T, ctx, bs=256, nkv=4, D=128, layers=2, kv="bf16"):
    """A pool of random keys/values: bf16, or int8 ("int8": per-token-head scales,
    "int8-channel": per-channel read scales with two exact outlier dims per head)."""
    from b200moe.engine.kv_cache import KVPool
    nb = T * math.ceil(ctx / bs)
    int8 = kv != "bf16"
    pool = KVPool(nb + 1, layers, nkv, bs, D, torch.bfloat16, "cuda", int8=int8,
                  int8_mode="channel" if kv == "int8-channel" else "token")
    if int8:
        pool.data.copy_(torch.randint(-127, 128, pool.data.shape, dtype=torch.int8, device="cuda"))
        if pool.scales is not None:
            pool.scales.uniform_(0.005, 0.02)
        else:
            pool.ch_dscale.uniform_(0.005, 0.02)
            pool.out_idx[:, :, :2] = torch.tensor([3, 77], dtype=torch.int32, device="cuda")
            pool.n_out.fill_(2)
            pool.side.normal_()
    else:
        pool.data.normal_()
    tables = torch.arange(nb, dtype=torch.int32, device="cuda").view(T, -1)
    return pool, tables


def case_decode(T, ctx, iters, nq=32, nkv=4, D=128, splits=0, pool_layers=2, kv="bf16"):
    """pool_layers: layers interleaved in each KV block slab (the engine's pool
    holds every layer of a block in one slab, so one layer's keys are strided).
    Bytes are the pool bytes read: 2 per value for bf16, 1 for int8."""
    from b200moe.models.qwen3_moe import Qwen3MoeForCausalLM
    pool, tables = _kv(T, ctx, layers=pool_layers, kv=kv)
    q = torch.randn(T, nq, D, device="cuda").to(torch.bfloat16)
    lens = torch.full((T,), ctx, dtype=torch.int32, device="cuda")
    out = torch.empty_like(q)
    model = type("M", (), {"args": type("A", (), {"num_key_value_heads": nkv})()})()
    split_len, nsplit = Qwen3MoeForCausalLM.decode_splits(model, T, ctx)
    if splits:
        per = -(-ctx // splits)
        split_len = -(-per // 64) * 64
        nsplit = -(-ctx // split_len)
    ws = (torch.empty(T * nq * nsplit, D, device="cuda"), torch.empty(T * nq * nsplit, device="cuda"),
          torch.empty(T * nq * nsplit, device="cuda"))
    ms = timeit(lambda: ops.decode_attention(q, pool.layer(0), tables, lens, D ** -0.5, out, split_len, nsplit, ws),
                iters)
    report("decode_attn", ms, T * ctx * nkv * D * 2 * (1 if kv != "bf16" else 2), 4 * T * ctx * nq * D, seqs=T,
           ctx=ctx, splits=nsplit, pool_layers=pool_layers, kv=kv)


def case_prefill(T, ctx, iters, nq=32, nkv=4, D=128, kv="bf16"):
    B = max(1, T // ctx)
    pool, tables = _kv(B, ctx, kv=kv)
    q = torch.randn(B * ctx, nq, D, device="cuda").to(torch.bfloat16)
    cu = torch.arange(0, B * ctx + 1, ctx, dtype=torch.int32, device="cuda")
    lens = torch.full((B,), ctx, dtype=torch.int32, device="cuda")
    out = torch.empty_like(q)
    ms = timeit(lambda: ops.prefill_attention(q, pool.layer(0), cu, lens, tables, ctx, D ** -0.5, out), iters)
    report("prefill_attn", ms, 0, 2 * B * ctx * ctx * nq * D, seqs=B, ctx=ctx, kv=kv)


def case_step(T, ctx, iters, layers=48):
    from b200moe.config import ModelArgs
    from b200moe.engine.kv_cache import KVPool
    from b200moe.models.qwen3_moe import Qwen3MoeForCausalLM, StepInputs
    from b200moe.utils.weights import random_init_
    args = ModelArgs(num_hidden_layers=layers)
    model = Qwen3MoeForCausalLM(args, "cuda")
    random_init_(model)
    if os.environ.get("B200MOE_TILED_WEIGHTS", "1") != "0":
        model.tile_weights_()
    bs = 256
    nbs = math.ceil((ctx + 1) / bs)
    model.reserve_workspace(max(T, 1), T, 64)
    pool = KVPool(T * nbs + 1, layers, 4, bs, 128, torch.bfloat16, "cuda")
    tables = torch.arange(T * nbs, dtype=torch.int32, device="cuda").view(T, -1)
    i32 = lambda t: t.to(torch.int32)
    pos = torch.full((T,), ctx, dtype=torch.int32, device="cuda")
    slots = i32(tables[:, ctx // bs] * bs + ctx % bs)
    inp = StepInputs(i32(torch.randint(0, 151936, (T,), device="cuda")), pos, slots,
                     torch.arange(T + 1, dtype=torch.int32, device="cuda"), pos + 1, tables,
                     torch.arange(T, dtype=torch.int32, device="cuda"), T, 0, ctx + 1, T)
    fn = lambda: model.compute_logits(model(inp, pool))
    ms = timeit(fn, iters, flush=False, reps=1)
    wbytes = layers * (128 * 3 * 2048 * 768 + (5120 + 2048) * 2048 * 1.0) + 151936 * 2048 * 2
    kvbytes = T * (ctx + 1) * layers * 4 * 128 * 2 * 2
    report("decode_step", ms, wbytes + kvbytes, 0, rows=T, ctx=ctx, layers=layers)


def case_ops(T, iters, H=2048, nq=32, nkv=4, D=128, V=151936, topk=8):
    """The memory-bound hot ops of a decode step at T rows, each timed alone (CUDA
    events, L2 flushed before every call); bytes are what each op must move:
    residual add + RMSNorm, q/k RMSNorm + RoPE + paged KV store, the MoE combine
    (fixed-order top-k sum + residual + next RMSNorm), greedy argmax and the sampler
    (temperature 0.7 with top-k 50 + top-p 0.9, and top-p 0.9 alone) over the full
    151,936-token vocabulary."""
    from b200moe.engine.kv_cache import KVPool
    dev = "cuda"
    bf = torch.bfloat16
    x = torch.randn(T, H, device=dev).to(bf)
    res = torch.randn(T, H, device=dev).to(bf)
    w = (1 + 0.1 * torch.randn(H, device=dev)).to(bf)
    out = torch.empty(T, H, device=dev, dtype=bf)
    ms = timeit(lambda: ops.rmsnorm(x, w, 1e-6, residual=res, out=out), iters)
    report("rmsnorm_residual", ms, 4 * T * H * 2, 0, rows=T, hidden=H)
    width = (nq + 2 * nkv) * D
    qkv = torch.randn(T, width, device=dev).to(bf)
    bs = 256
    pool = KVPool(T // 4 + 2, 2, nkv, bs, D, bf, dev)
    slots = torch.randperm((T // 4 + 1) * bs, device=dev)[:T].to(torch.int32)
    pos = torch.randint(0, 4000, (T,), dtype=torch.int32, device=dev)
    qw = (1 + 0.1 * torch.randn(D, device=dev)).to(bf)
    kw = (1 + 0.1 * torch.randn(D, device=dev)).to(bf)
    cs = ops.rope_cos_sin(D, 4096, 1e6, dev)
    q_out = torch.empty(T, nq, D, device=dev, dtype=bf)
    ms = timeit(lambda: ops.qknorm_rope_kvstore(qkv, pos, slots, qw, kw, cs, pool.layer(1), nq, nkv, D, 1e-6,
                                                q_out=q_out), iters)
    report("qknorm_rope_kvstore", ms, T * width * 2 + T * (nq + 2 * nkv) * D * 2, 0, rows=T)
    slot_buf = torch.randn(T * topk, H, device=dev).to(bf)
    ms = timeit(lambda: ops.moe_combine_add_rmsnorm(slot_buf, topk, res, w, 1e-6, out=out), iters)
    report("moe_combine_add_rmsnorm", ms, (T * topk * H + 3 * T * H) * 2, 0, rows=T, topk=topk)
    logits = torch.randn(T, V, device=dev)
    tok = torch.empty(T, dtype=torch.int32, device=dev)
    ms = timeit(lambda: ops.argmax(logits, tok), iters)
    report("argmax", ms, T * V * 4, 0, rows=T, vocab=V)
    temp = torch.full((T,), 0.7, device=dev)
    top_k = torch.full((T,), 50, dtype=torch.int32, device=dev)
    top_p = torch.full((T,), 0.9, device=dev)
    seeds = torch.arange(T, dtype=torch.int64, device=dev)
    ms = timeit(lambda: ops.sample(logits, temp, top_k, top_p, None, seeds, None, out=tok), iters)
    report("sample_topk_topp", ms, T * V * 4, 0, rows=T, vocab=V)
    no_k = torch.full((T,), -1, dtype=torch.int32, device=dev)
    ms = timeit(lambda: ops.sample(logits, temp, no_k, top_p, None, seeds, None, out=tok), iters)
    report("sample_topp", ms, T * V * 4, 0, rows=T, vocab=V)


NVLINK_GBS = 770.0  # measured peer copy per direction on this pool's NVSwitch systems


def case_ep(T, iters, reps=10):
    """One expert-parallel MoE layer of Qwen3-30B-A3B on every rank of a torchrun job
    (``torchrun --nproc-per-node W -m b200moe.microbench ep --tokens T``): router,
    dispatch, scatter, grouped GEMMs, peer-scatter combine -- the fused peer-memory
    path, ``reps`` layers (each with its own weights) per CUDA graph, device time max
    over ranks.  The roofline
    is the slowest of: NVLink bytes (rows out + weighted rows back) at the measured
    peer bandwidth, this rank's expert weights at the measured HBM copy rate, and
    the expert FLOPs at the measured bf16 peak."""
    from types import SimpleNamespace

    import torch.distributed as dist

    from b200moe.config import Config
    from b200moe.engine.model_runner import expert_placement
    from b200moe.models.qwen3_moe import Qwen3MoeForCausalLM
    from b200moe.parallel.ep import ExpertParallel
    from b200moe.utils.weights import random_init_
    rank, W = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev)
    cfg = Config("qwen3-30b-a3b", max_num_batched_tokens=max(T, 16), max_num_seqs=max(T, 1))
    args = cfg.hf_config
    # one layer per rep: every rep reads its own expert weights from HBM (at 8 ranks one layer's
    # 38 MB slice would otherwise stay in the 126 MB L2 across reps)
    args.num_hidden_layers = reps
    model = Qwen3MoeForCausalLM(args, dev, ep_rank=rank, ep_size=W, expert_ids=expert_placement(cfg, rank, W))
    random_init_(model, seed=7)
    model.tile_weights_()
    model.reserve_workspace(max(T, 16), max(T, 1), 8)
    runner = SimpleNamespace(world_size=W, rank=rank, device=dev, args=args, config=cfg, model=model)
    ep = ExpertParallel(runner, "fused")
    assert ep.backend == "fused"
    model.ep = ep
    g = torch.Generator(device=dev).manual_seed(rank)
    x = (torch.randn(T, args.hidden_size, device=dev, generator=g)).to(torch.bfloat16)
    res0 = torch.randn(T, args.hidden_size, device=dev, generator=g).to(torch.bfloat16)
    res = res0.clone()

    def fn():
        for layer in model.layers:
            model._mlp(layer, x, res, model.norm, T)

    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    graph = _graph(fn, 1)
    dist.barrier()
    ms = _time_graph(graph, iters) / reps
    ms_max = torch.tensor([ms], device=dev)
    dist.all_reduce(ms_max, op=dist.ReduceOp.MAX)
    ms = float(ms_max)
    k, H, I = args.num_experts_per_tok, args.hidden_size, args.moe_intermediate_size
    nvlink = 2 * T * k * H * 2 * (W - 1) / W               # bf16 rows to the owners and back, per rank
    wbytes = model.num_local_experts * 3 * H * I            # e4m3 expert weights of this rank
    flops = 2 * T * k * H * 3 * I                           # gate, up and down of the rows this rank receives
    bw, tf, src = peaks()
    t_link, t_hbm, t_tc = nvlink / (NVLINK_GBS * 1e9), wbytes / bw, flops / tf
    roof = max(t_link, t_hbm, t_tc)
    waits = ep.p2p.wait_stats()
    if rank == 0:
        print(json.dumps({"kernel": "ep_moe_layer", "world": W, "tokens_per_rank": T, "ms": round(ms, 4),
                          "roofline_ms": round(roof * 1e3, 4), "roofline_frac": round(roof / (ms / 1e3), 3),
                          "bound": ["nvlink", "hbm", "tensor"][[t_link, t_hbm, t_tc].index(roof)],
                          "nvlink_bytes": int(nvlink), "weight_bytes": int(wbytes), "flops": int(flops),
                          "peak": src, "nvlink_gbs": NVLINK_GBS,
                          "wait_ms_rank0_over_run": waits}), flush=True)
    model.ep = None
    del graph
    ep.p2p.close()
    dist.destroy_process_group()


def case_tp(T, iters, reps=10, H=2048, K_total=4096):
    """Tensor-parallel O projection + sum over ranks + residual RMSNorm for T tokens on
    every rank of a torchrun job (``--nproc-per-node W -m b200moe.microbench tp``):
    the fused peer-memory path (parallel/tp.py) against the NCCL path (GEMM,
    all-reduce, RMSNorm), ``reps`` calls per CUDA graph, max over ranks.  The fused
    path's roofline is the slowest of this rank's e4m3 weight slice at the measured
    HBM rate and the (W-1) fp32 partials it reads over NVLink."""
    from types import SimpleNamespace

    import torch.distributed as dist

    from b200moe.parallel.tp import TpComm
    from b200moe.utils.weights import quantize_block_fp8
    rank, W = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev)
    K = K_total // W
    runner = SimpleNamespace(world_size=W, rank=rank, device=dev, args=SimpleNamespace(hidden_size=H),
                             config=SimpleNamespace(max_num_batched_tokens=max(T, 16)))
    tp = TpComm.create(runner)
    assert tp is not None
    g = torch.Generator(device=dev).manual_seed(rank)
    q, sc = quantize_block_fp8(torch.randn(1, H, K, device=dev, generator=g) * 0.02)
    w8 = ops.tile_fp8(q[0])
    x = torch.randn(T, K, device=dev, generator=g).to(torch.bfloat16)
    res = torch.randn(T, H, device=dev).to(torch.bfloat16)
    nw = torch.ones(H, device=dev, dtype=torch.bfloat16)
    out = torch.empty(T, H, device=dev, dtype=torch.bfloat16)
    o = torch.empty(T, H, device=dev, dtype=torch.bfloat16)

    def fused():
        tp.begin_forward(1)
        tp.o_proj_add_norm(x, w8, sc[0], res, nw, 1e-6, out, True)

    def nccl():
        ops.linear(x, w8, sc[0], out=o, tiled=True)
        dist.all_reduce(o)
        ops.rmsnorm(o, nw, 1e-6, residual=res, out=out)

    def fused_gemm():  # the O GEMM alone, writing its peer-visible partials and releasing
        T_, K_ = x.shape
        bn, splits = ops.plan_dense(T_, H // 128, K_ // 64, fp8=True, max_splits=4)
        part = tp.part[0][0][:splits * T_].view(splits * T_, H)
        release = [tp.epoch.data_ptr(), tp.prod_counter.data_ptr(), tp.rank, 1, *tp.flag_ptrs]
        ops.native().gemm(w8, sc[0], x, ops.count_tensor(T_, dev), None, part, bn, ops.EPI_F32, H // 128,
                          0, 0, None, None, tp.status, ops._trace[0], splits, T_ * H, True, release)

    def linear():
        ops.linear(x, w8, sc[0], out=o, tiled=True)

    times = {}
    for name, fn in (("fused", fused), ("nccl", nccl), ("fused_gemm", fused_gemm), ("linear", linear)):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        graph = _graph(fn, reps)
        dist.barrier()
        t = torch.tensor([_time_graph(graph, iters) / reps], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        times[name] = float(t)
        del graph
    bw, tf, src = peaks()
    wbytes = H * K                                   # this rank's e4m3 O slice
    nvlink = (W - 1) * T * H * 4                     # fp32 partials read from every peer
    roof = max(wbytes / bw, nvlink / (NVLINK_GBS * 1e9), 2 * T * H * K / tf)
    if rank == 0:
        print(json.dumps({"kernel": "tp_o_proj_allreduce_norm", "world": W, "tokens": T,
                          "fused_ms": round(times["fused"], 4), "nccl_ms": round(times["nccl"], 4),
                          "fused_gemm_ms": round(times["fused_gemm"], 4), "linear_ms": round(times["linear"], 4),
                          "roofline_ms": round(roof * 1e3, 4), "fused_roofline_frac": round(roof * 1e3 / times["fused"], 3),
                          "nvlink_bytes": nvlink, "weight_bytes": wbytes, "peak": src,
                          "wait_ms_rank0": tp.wait_stats()}), flush=True)
    tp.close()
    dist.destroy_process_group()


def _trace_summary(name, buf):
    import statistics
    cap = (buf.numel() - 1) // 10
    slots = buf[1:1 + 10 * cap].view(10, cap).tolist()
    by = {r: {i: t for i, t in enumerate(row) if t} for r, row in enumerate(slots)}
    med = lambda xs: round(statistics.median(xs) / 1e3, 3) if xs else None
    issue, c0, c1, mma = (by.get(r, {}) for r in (0, 1, 2, 3))
    idx = sorted(set(issue) & set(c0) & set(c1) & set(mma)) or sorted(set(issue) & set(mma))
    d = {"kernel": name, "stages_traced": len(idx)}
    if os.environ.get("B200MOE_TRACE_DUMP") and idx:
        # stage timeline (us from the first issue): producer reaches, A slot free, issued, landed,
        # dequant start/end, MMA thread reaches, MMA issued
        t0 = min(issue.values())
        for i in idx[40:72]:
            row = [round((r[i] - t0) / 1e3, 2) if i in r else None
                   for r in (by.get(7, {}), by.get(8, {}), issue, by.get(6, {}), c0, c1, by.get(9, {}), mma)]
            print(json.dumps({"trace": name, "stage": i, "t": row}))
    if len(idx) > 2:
        d["us_between_tma_issues"] = med([issue[b] - issue[a] for a, b in zip(idx, idx[1:])])
        d["us_between_mma_issues"] = med([mma[b] - mma[a] for a, b in zip(idx, idx[1:])])
        landed = by.get(6, {})
        if landed and all(i in landed for i in idx):
            d["us_issue_to_landed"] = med([landed[i] - issue[i] for i in idx])
            d["us_landed_to_dequant_start"] = med([c0[i] - landed[i] for i in idx])
        if c0:
            d["us_issue_to_dequant_start"] = med([c0[i] - issue[i] for i in idx])
            d["us_dequant"] = med([c1[i] - c0[i] for i in idx])
            d["us_dequant_done_to_mma"] = med([mma[i] - c1[i] for i in idx])
        else:
            d["us_issue_to_mma"] = med([mma[i] - issue[i] for i in idx])
    e0, e1 = by.get(4, {}), by.get(5, {})
    tiles = sorted(set(e0) & set(e1))
    allt = [t for r in by.values() for t in r.values()]
    if allt:
        d["us_cta0_span"] = round((max(allt) - min(allt)) / 1e3, 2)
    if len(tiles) > 2:
        d["us_per_tile"] = med([e0[b] - e0[a] for a, b in zip(tiles, tiles[1:])])
    if tiles:
        d["tiles"] = len(tiles)
        d["us_epilogue"] = med([e1[i] - e0[i] for i in tiles])
    print(json.dumps(d), flush=True)


def case_trace(T):
    """Per-stage timeline of CTA 0 for the decode-size GEMMs."""
    buf = torch.zeros(1 + 10 * 4096, dtype=torch.int64, device="cuda")
    H, I, E, k = 2048, 768, 128, 8
    x = (torch.randn(T, 4096, device="cuda") * 0.5).to(torch.bfloat16)
    q, s = fp8_weight(1, H, 4096, 4)
    q = ops.tile_fp8(q) if TILED else q
    for name, fn in (("o_proj", lambda: ops.linear(x, q[0], s[0], tiled=TILED)),):
        fn()
        torch.cuda.synchronize()
        buf.zero_()
        ops.set_gemm_trace(buf)
        flush_l2()
        fn()
        torch.cuda.synchronize()
        ops.set_gemm_trace(None)
        _trace_summary(name, buf.cpu())
    q13, s13 = fp8_weight(E, 2 * I, H, 1)
    q13 = ops.tile_fp8(q13) if TILED else q13
    rows = T * k
    ids = torch.stack([torch.randperm(E, device="cuda")[:k] for _ in range(T)]).flatten()
    counts = torch.bincount(ids, minlength=E).to(torch.int32)
    offsets = torch.zeros(E + 1, dtype=torch.int32, device="cuda")
    offsets[1:] = torch.cumsum(counts, 0)
    xm = (torch.randn(rows, H, device="cuda") * 0.5).to(torch.bfloat16)
    h = torch.empty(rows, I, dtype=torch.bfloat16, device="cuda")
    q2, s2 = fp8_weight(E, H, I, 2)
    q2 = ops.tile_fp8(q2) if TILED else q2
    slots = torch.empty(rows, H, dtype=torch.bfloat16, device="cuda")
    sor = torch.randperm(rows, device="cuda").to(torch.int32)
    w = torch.rand(rows, device="cuda")
    for name, fn in (("moe_gate_up", lambda: ops.grouped_gate_up_silu(xm, q13, s13, counts, offsets, h, I,
                                                                      tiled=TILED)),
                     ("moe_down", lambda: ops.grouped_down_scatter(h, q2, s2, counts, offsets, sor, w, slots,
                                                                   tiled=TILED))):
        fn()
        torch.cuda.synchronize()
        buf.zero_()
        ops.set_gemm_trace(buf)
        flush_l2()
        fn()
        torch.cuda.synchronize()
        ops.set_gemm_trace(None)
        _trace_summary(name, buf.cpu())


def main():
    p = argparse.ArgumentParser()
    p.add_argument("case", choices=["moe", "dense", "decode", "prefill", "step", "trace", "ep", "tp", "ops", "all"])
    p.add_argument("--tokens", type=int, default=256)
    p.add_argument("--ctx", type=int, default=1152)
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--layers", type=int, default=48)
    p.add_argument("--splits", type=int, default=0, help="decode: force this many KV splits (0 = heuristic)")
    p.add_argument("--pool-layers", type=int, default=2, help="decode: layers per KV block slab")
    p.add_argument("--only", choices=["", "gate_up", "down"], default="", help="moe: time one of the two GEMMs")
    p.add_argument("--kv", choices=["bf16", "int8", "int8-channel"], default="bf16", help="decode / prefill: pool type")
    a = p.parse_args()
    if a.case == "ep":
        return case_ep(a.tokens, a.iters)
    if a.case == "tp":
        return case_tp(a.tokens, a.iters)
    torch.cuda.set_device(0)
    if a.case in ("moe", "all"):
        case_moe(a.tokens, a.iters, only=a.only)
    if a.case in ("dense", "all"):
        case_dense(a.tokens, a.iters)
    if a.case in ("decode", "all"):
        case_decode(a.tokens, a.ctx, a.iters, splits=a.splits, pool_layers=a.pool_layers, kv=a.kv)
    if a.case in ("prefill", "all"):
        case_prefill(max(a.tokens, a.ctx), a.ctx, a.iters, kv=a.kv)
    if a.case == "trace":
        case_trace(a.tokens)
    if a.case == "step":
        case_step(a.tokens, a.ctx, a.iters, a.layers)
    if a.case in ("ops", "all"):
        case_ops(a.tokens, a.iters)
    ops.check_status("cuda")


if __name__ == "__main__":
    main()
