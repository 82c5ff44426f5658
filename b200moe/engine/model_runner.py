"""Per-rank device runtime: model, KV pool, step upload, CUDA graphs, sampling.

One ``ModelRunner`` lives in each rank's process and owns that rank's GPU.  A
step arrives as a :class:`StepPlan`; the runner packs it into one pinned int32
buffer, issues ONE host-to-device copy, runs the forward (a captured CUDA graph
for pure-decode steps up to ``cuda_graph_max_bs`` rows, eager otherwise),
samples on the device and returns the sampled ids with a single
device-to-host read.

Reference: nanovllm/engine/model_runner.py:95-1248 (pickled Sequence objects,
per-tensor pinned copies, whole-graph capture per batch bucket).
"""
from __future__ import annotations

import collections
import gc
import math
import os
import time

import numpy as np
import torch
import torch.distributed as dist

from b200moe import ops
from b200moe.config import Config
from b200moe.engine.kv_cache import KVPool
from b200moe.engine.step_plan import StepPlan, empty_plan, pack_plan, pack_sampling, validate_plan
from b200moe.models.qwen3_moe import Qwen3MoeForCausalLM, StepInputs
from b200moe.utils.init_trace import InitTrace
from b200moe.utils.profiler import DeviceProfiler
from b200moe.utils.weights import load_checkpoint, random_init_

GRAPH_BUCKETS = (1, 2, 4, 8, 16, 24, 32, 48, 64, 96, 128, 160, 192, 224, 256, 320, 384, 448, 512)


def expert_placement(config: Config, rank: int, world: int, layer: int = 0) -> list[int]:
    """Global expert ids owned by ``rank`` (reference: qwen3_moe.py:144-166)."""
    E = config.hf_config.num_experts
    per = E // world
    if config.expert_placement == "linear":
        return list(range(rank * per, (rank + 1) * per))
    if config.expert_placement == "round_robin":
        return list(range(rank, E, world))
    import hashlib
    import json
    with open(config.expert_map_path) as f:
        mapping = json.load(f)
    want = mapping.get("model_config_sha256")
    if want and os.path.isdir(config.model):
        with open(os.path.join(config.model, "config.json"), "rb") as f:
            got = hashlib.sha256(f.read()).hexdigest()
        if got != want:
            raise ValueError("profiled expert map was generated for a different model config")
    layers = mapping.get("layers", mapping)
    lm = layers.get(str(layer), layers.get(layer))
    ids = lm.get(str(rank), lm.get(rank))
    if len(ids) != per or len(set(ids)) != per:
        raise ValueError("profiled expert map must give each rank E/world distinct experts")
    return list(ids)


class ModelRunner:

    def __init__(self, config: Config, rank: int = 0, world_size: int | None = None, init_dist: bool = True):
        self.config = config
        self.rank = rank
        trace = InitTrace(rank)
        self.world_size = world_size or config.world_size
        self.block_size = config.kvcache_block_size
        args = config.hf_config
        self.args = args
        if config.device == "cuda":
            if not torch.cuda.is_available():
                raise RuntimeError("device='cuda' but no CUDA device is visible")
            local = rank % torch.cuda.device_count()
            torch.cuda.set_device(local)
            self.device = torch.device("cuda", local)
            ops.native()  # fail loudly when the extension is missing on a GPU box
        else:
            self.device = torch.device("cpu")
        trace.mark("device")
        if self.world_size > 1 and init_dist:
            self._init_dist()
            trace.mark("process_group")
        self.profiler = DeviceProfiler(self.device, enabled=config.enable_profiling)
        expert_ids = expert_placement(config, rank, self.world_size) if args.is_moe else []
        t0 = time.perf_counter()
        # tensor-parallel attention: heads split over the ranks, every rank sees every token
        self.attn_tp = self.world_size if (config.attention_parallel == "tp" and self.world_size > 1) else 1
        self.model = Qwen3MoeForCausalLM(args, self.device, ep_rank=rank, ep_size=self.world_size,
                                         expert_ids=expert_ids, attn_tp=self.attn_tp, attn_rank=rank)
        self.model.moe_backend = "loop" if config.moe_backend == "loop" else "fused"
        self.model.attention_backend = config.attention_backend
        if self.world_size > 1 and self.attn_tp == 1:
            from b200moe.parallel.ep import ExpertParallel
            self.model.ep = ExpertParallel(self, config.moe_backend)
        if self.attn_tp > 1 and self.device.type == "cuda":
            from b200moe.parallel.tp import TpComm
            self.model.tp_comm = TpComm.create(self)
        trace.mark("model")
        if config.random_init:
            random_init_(self.model, seed=config.seed)
        else:
            load_checkpoint(self.model, config.model)
        trace.mark("weights")
        if os.environ.get("B200MOE_TILED_WEIGHTS", "1") != "0":
            self.model.tile_weights_()  # e4m3 GEMM weights tile-major: one contiguous HBM block per stage
            trace.mark("tile_weights")
        self.model.profiler = self.profiler if config.enable_profiling else None
        self.bf16_expert_cache_bytes = self._maybe_cache_bf16_experts()
        self.load_s = time.perf_counter() - t0
        self.max_blocks = -(-config.max_model_len // self.block_size)
        self.max_rows = config.max_num_seqs
        self.max_tokens = config.max_num_batched_tokens
        self.max_splits = self.model.decode_splits(1, config.max_model_len)[1]
        if self.device.type == "cuda":
            self.model.reserve_workspace(self.max_tokens, self.max_rows, self.max_splits)
            trace.mark("workspace")
        self.allocate_kv_cache()
        trace.mark("kv_cache")
        # two pinned staging buffers: a step may be uploaded while the previous one's copy is in flight
        words = 8 * self.max_tokens + 8 * self.max_rows + self.max_rows * self.max_blocks + 16
        pin = self.device.type == "cuda"
        self._pinned = [torch.empty(words, dtype=torch.int32, pin_memory=pin) for _ in range(2)]
        self._pinned_np = [p.numpy() for p in self._pinned]
        self._dev_in = torch.empty(words, dtype=torch.int32, device=self.device)
        # the last step's sampled tokens (plan-row order), read by the next step's
        # embedding for rows launched before the host collected them
        self._feed_tokens = torch.zeros(max(self.max_rows, 1), dtype=torch.int32, device=self.device)
        # sampling arrays of a step (pack_sampling): two pinned staging buffers, one device buffer, grown on demand
        self._samp_pinned = [torch.empty(16 * max(self.max_rows, 1), dtype=torch.int32, pin_memory=pin)
                             for _ in range(2)]
        self._samp_pinned_np = [p.numpy() for p in self._samp_pinned]
        self._samp_dev = torch.empty(16 * max(self.max_rows, 1), dtype=torch.int32, device=self.device)
        self._samp_idx = 0
        self._pin_idx = 0
        self._validate = os.environ.get("B200MOE_VALIDATE_PLANS", "1") != "0"
        self._logits = None
        self.graphs: dict[int, tuple] = {}
        self.graph_pool = None
        self.offloader = None
        self._pending: collections.deque = collections.deque()  # steps launched, not yet collected
        self.steps = 0
        self.h2d_bytes = 0
        self._step_events: list = []
        self._graph_kernels: dict[int, int] = {}
        if self._graphs_allowed():
            self.capture_cudagraphs()
            trace.mark("cuda_graphs")
        self.init_stages = trace.done()

    def _graphs_allowed(self) -> bool:
        """Decode graphs need the native paths: the per-expert loop and the
        PyTorch attention read counts back to the host."""
        ep_ok = self.model.ep is None or self.model.ep.graph_safe
        return (self.device.type == "cuda" and not self.config.enforce_eager and ep_ok
                and self.model.moe_backend == "fused" and self.model.attention_backend == "paged")

    def _set_backend(self, attr: str, value: str):
        if getattr(self.model, attr) == value:
            return
        setattr(self.model, attr, value)
        self.graphs.clear()
        self._graph_kernels.clear()
        self.graph_pool = None
        if self._graphs_allowed():
            self.capture_cudagraphs()

    def set_moe_backend(self, backend: str):
        """Switch between the native grouped path ("fused") and the per-expert
        PyTorch loop ("loop", the A/B and equivalence baseline) between steps."""
        if backend not in ("fused", "loop"):
            raise ValueError("runtime MoE backend must be 'fused' or 'loop'")
        if backend == "loop" and self.model.ep is not None:
            raise ValueError("the per-expert loop runs on one rank only")
        self._set_backend("moe_backend", backend)

    def set_cuda_graphs(self, enabled: bool):
        """Turn decode CUDA graphs on or off between steps (graph A/B runs)."""
        self.config.enforce_eager = not enabled
        self.graphs.clear()
        self._graph_kernels.clear()
        self.graph_pool = None
        if self._graphs_allowed():
            self.capture_cudagraphs()

    def kv_heads(self) -> int:
        return self.kv.num_kv_heads

    def memory_reserved(self) -> int:
        return torch.cuda.memory_reserved(self.device) if self.device.type == "cuda" else 0

    @torch.inference_mode()
    def score_tokens(self, token_ids: list[int]) -> torch.Tensor:
        """Teacher-forced logits [L, V] (fp32, host) at every position of one
        sequence, prefilled from scratch.  It writes KV blocks 0..ceil(L/bs)-1,
        so call it only while no request holds KV, and clear the prefix cache
        afterwards (those blocks may back cached prefixes)."""
        L = len(token_ids)
        nb = -(-L // self.block_size)
        if L == 0 or L > self.max_tokens or nb > self.max_blocks:
            raise ValueError("sequence longer than max_num_batched_tokens / max_model_len")
        ids = np.asarray(token_ids, np.int32)
        pos = np.arange(L, dtype=np.int32)
        tables = np.zeros((1, self.max_blocks), np.int32)
        tables[0, :nb] = np.arange(nb, dtype=np.int32)
        plan = StepPlan(ids, pos, pos.copy(), np.array([0, L], np.int32), np.array([L], np.int32), tables, 0, L, L,
                        np.zeros(1, np.int32), np.zeros(1, np.float32))
        inp = self._inputs(plan, self._upload(plan))
        inp.logits_indices = torch.arange(L, dtype=torch.int32, device=self.device)
        h = self.model(inp, self.kv)
        return self.model.compute_logits(h).float().cpu()

    def set_attention_backend(self, backend: str):
        """"paged" (native kernels) or "sdpa" (per-sequence PyTorch attention
        over the same paged pool, fp32 math)."""
        if backend not in ("paged", "sdpa"):
            raise ValueError("attention backend must be 'paged' or 'sdpa'")
        self._set_backend("attention_backend", backend)

    # ------------------------------------------------------------- setup
    def _init_dist(self):
        import torch.distributed as dist
        from datetime import timedelta
        if not dist.is_initialized():
            backend = "nccl" if self.device.type == "cuda" else "gloo"
            method = self.config.distributed_init_method or "env://"
            dist.init_process_group(backend, init_method=method, world_size=self.world_size, rank=self.rank,
                                    timeout=timedelta(seconds=self.config.rank_timeout_s),
                                    device_id=self.device if self.device.type == "cuda" else None)

    # Resident bf16 copy of this rank's expert weights for prefill-size steps (the
    # single-GPU expert path and the fused expert-parallel path): "auto" keeps it when at
    # least this fraction of the GPU's memory stays free for the KV cache afterwards;
    # "1" always, "0" never (B200MOE_BF16_EXPERT_CACHE).
    BF16_CACHE_KEEP_FREE = 0.35

    def _maybe_cache_bf16_experts(self) -> int:
        mode = os.environ.get("B200MOE_BF16_EXPERT_CACHE", "auto")
        m = self.model
        if (mode == "0" or self.device.type != "cuda" or m.attn_tp > 1 or m.BF16_EXPERT_ROWS <= 0
                or (m.ep is not None and m.ep.backend != "fused")):
            return 0
        need = m.bf16_expert_bytes()
        if need == 0:
            return 0
        free, total = torch.cuda.mem_get_info(self.device)
        if mode != "1" and free - need < self.BF16_CACHE_KEEP_FREE * total:
            return 0
        return m.cache_bf16_experts_()

    def allocate_kv_cache(self):
        c, a = self.config, self.args
        int8 = c.kv_cache_dtype == "int8"
        nkv = self.model.nkv_local
        block_bytes = KVPool.bytes_per_block(a.num_hidden_layers, nkv, self.block_size, a.head_dim,
                                             self.model.dtype, int8, c.kv_int8_mode)
        if c.num_kvcache_blocks <= 0:
            if self.device.type == "cuda":
                free, total = torch.cuda.mem_get_info(self.device)
                reserve = 3 << 30  # graphs, logits, transient allocator growth
                if int8:
                    reserve += ops.INT8_STAGE_MAX_BYTES  # bf16 staging of int8 blocks for the prefill kernel
                budget = free - (1.0 - c.gpu_memory_utilization) * total - reserve
                c.num_kvcache_blocks = int(budget // block_bytes)
            else:
                c.num_kvcache_blocks = max(64, c.max_num_seqs * self.max_blocks // 4)
        if self.world_size > 1:
            import torch.distributed as dist
            t = torch.tensor([c.num_kvcache_blocks], dtype=torch.int64, device=self.device)
            dist.all_reduce(t, op=dist.ReduceOp.MIN)
            c.num_kvcache_blocks = int(t.item())
        if c.num_kvcache_blocks <= 0:
            raise RuntimeError(f"no memory left for the KV cache (block = {block_bytes / 2**20:.1f} MiB)")
        self.kv = KVPool(c.num_kvcache_blocks + 1, a.num_hidden_layers, nkv, self.block_size, a.head_dim,
                         self.model.dtype, self.device, int8=int8, int8_mode=c.kv_int8_mode)
        self._calib_tokens = None  # int8 channel mode: tokens stored while calibrating
        self.block_bytes = block_bytes
        self.scratch_block = self.kv.scratch_block

    # ------------------------------------------------------------ upload
    def _upload(self, plan: StepPlan, dev: torch.Tensor | None = None) -> dict:
        i = self._pin_idx
        self._pin_idx ^= 1
        buf, offs = pack_plan(plan, self._pinned_np[i])
        n = buf.size
        self.h2d_bytes += 4 * n
        dev = self._dev_in if dev is None else dev
        if n > dev.numel():
            raise RuntimeError("step plan larger than the staging buffer")
        dev[:n].copy_(self._pinned[i][:n], non_blocking=True)
        views = {k: dev[o:o + s] for k, (o, s) in offs.items()}
        views["block_tables"] = views["block_tables"].view(plan.num_rows, plan.block_tables.shape[1])
        return views

    def _inputs(self, plan: StepPlan, v: dict, max_seq_len: int | None = None, feed: bool = False) -> StepInputs:
        nd = plan.num_decode
        return StepInputs(
            input_ids=v["input_ids"], positions=v["positions"], slot_mapping=v["slot_mapping"],
            cu_seqlens_q=v["cu_seqlens_q"], seq_lens=v["seq_lens"], block_tables=v["block_tables"],
            logits_indices=v["logits_indices"], num_decode=nd, max_q_len=plan.max_q_len,
            max_seq_len=max_seq_len or plan.max_seq_len, num_rows=plan.num_rows,
            prefill_cu=v["prefill_cu"] if plan.num_rows > nd else None,
            feed_src=v["feed_src"] if (feed or plan.feed_src is not None) else None,
            feed_tokens=self._feed_tokens if (feed or plan.feed_src is not None) else None)

    def _pad_plan(self, plan: StepPlan, rows: int) -> StepPlan:
        """A decode plan padded to ``rows`` rows; padding rows write the scratch block."""
        B = plan.num_rows
        p = rows - B
        mb = self.max_blocks
        tables = np.full((rows, mb), self.scratch_block, np.int32)
        tables[:B, :plan.block_tables.shape[1]] = plan.block_tables
        tables[:B, plan.block_tables.shape[1]:] = 0
        pad_i = np.zeros(p, np.int32)
        feed = plan.feed_src if plan.feed_src is not None else np.full(B, -1, np.int32)
        return StepPlan(
            np.concatenate([plan.input_ids, pad_i]), np.concatenate([plan.positions, pad_i]),
            np.concatenate([plan.slot_mapping, np.full(p, self.scratch_block * self.block_size, np.int32)]),
            np.arange(rows + 1, dtype=np.int32), np.concatenate([plan.seq_lens, np.ones(p, np.int32)]),
            tables, rows, 0, plan.max_seq_len, np.arange(rows, dtype=np.int32),
            np.concatenate([plan.temperature, np.zeros(p, np.float32)]),
            feed_src=np.concatenate([feed, np.full(p, -1, np.int32)]))

    # ------------------------------------------------------------ graphs
    def _bucket(self, rows: int) -> int | None:
        for b in GRAPH_BUCKETS:
            if b >= rows and b <= min(self.config.cuda_graph_max_bs, self.max_rows):
                return b
        return None

    @torch.inference_mode()
    def capture_cudagraphs(self):
        """One graph per decode bucket: forward + LM head + greedy argmax into
        static buffers.  Decode split sizing uses max_model_len so the graph
        is valid for any context length.  Profiler ranges stay out of the
        graphs: a replayed step is timed as one "forward" range."""
        prof, self.model.profiler = self.model.profiler, None
        try:
            self._capture_cudagraphs()
        finally:
            self.model.profiler = prof

    def _capture_cudagraphs(self):
        max_bs = min(self.config.cuda_graph_max_bs, self.max_rows)
        buckets = [b for b in GRAPH_BUCKETS if b <= max_bs]
        V = self.args.vocab_size
        self._graph_logits = torch.empty(max(buckets), V, dtype=torch.float32, device=self.device)
        self._graph_tokens = torch.empty(max(buckets), dtype=torch.int32, device=self.device)
        words = self._dev_in.numel()
        self.graph_pool = torch.cuda.graph_pool_handle()
        stream = torch.cuda.Stream(self.device)
        for b in reversed(buckets):
            dummy = self._pad_plan(empty_plan(self.max_blocks), b)
            dummy.max_seq_len = self.config.max_model_len
            dev = torch.empty(words, dtype=torch.int32, device=self.device)
            views = self._upload(dummy, dev)
            inp = self._inputs(dummy, views, max_seq_len=self.config.max_model_len, feed=True)
            logits = self._graph_logits[:b]
            tokens = self._graph_tokens[:b]
            # warm-up run outside capture (first-use allocations, cached tensors).  With
            # expert parallelism it exchanges rows with every peer under bounded flag
            # waits: line the ranks up first, as start-up work before the first capture
            # (weight init, tiling, KV allocation) can leave them seconds apart.
            if (self.model.ep is not None or self.model.tp_comm is not None) and dist.is_initialized():
                torch.cuda.synchronize(self.device)
                dist.barrier()
            h = self.model(inp, self.kv)
            self.model.compute_logits(h, out=logits)
            ops.argmax(logits, tokens)
            torch.cuda.synchronize(self.device)
            g = torch.cuda.CUDAGraph()
            n0 = ops.launch_count()
            stream.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.graph(g, pool=self.graph_pool, stream=stream):
                h = self.model(inp, self.kv)
                self.model.compute_logits(h, out=logits)
                ops.argmax(logits, tokens)
            torch.cuda.synchronize(self.device)
            self._graph_kernels[b] = ops.launch_count() - n0
            self.graphs[b] = (g, dev, logits, tokens)
        ops.check_status(self.device)

    # --------------------------------------------------------------- run
    @torch.inference_mode()
    def run(self, plan: StepPlan):
        """Forward + sample; returns (token ids in plan-row order, logprobs|None)."""
        self.launch(plan)
        return self.collect()

    @torch.inference_mode()
    def launch(self, plan: StepPlan):
        """Enqueue the step (no host sync); ``collect`` reads the result."""
        if self._validate:
            validate_plan(plan, self.config.num_kvcache_blocks, self.block_size, self.args.vocab_size,
                          self._feed_tokens.numel())
        self.steps += 1
        B = plan.num_rows
        t_start = None
        if self.device.type == "cuda":
            t_start = torch.cuda.Event(enable_timing=True)
            t_start.record()
        if B == 0:
            if self.model.ep is not None:  # expert-parallel peers still need this rank's collectives
                self.model(self._inputs(plan, self._upload(plan)), self.kv)
            self._pending.append((plan, None, None))
            return
        bucket = self._bucket(B) if (plan.is_pure_decode and self.graphs) else None
        if bucket is not None:
            g, dev, logits, tokens = self.graphs[bucket]
            self._upload(self._pad_plan(plan, bucket), dev)
            g.replay()
            ops.count_launches(self._graph_kernels.get(bucket, 0))
            logits, tokens = logits[:B], tokens[:B]
        else:
            views = self._upload(plan)
            if self._calib_tokens is not None:
                self._calib_tokens += plan.num_tokens
            with self.profiler.range("forward"):
                h = self.model(self._inputs(plan, views), self.kv)
            logits = self.model.compute_logits(h)
            tokens = None
        lp = None
        if plan.needs_full_sampler or tokens is None:
            tokens, lp_dev = self._sample(plan, logits)
            if lp_dev is not None:  # log-probs ride the same device-to-host read as the tokens
                pin = self.device.type == "cuda"
                lp = tuple(torch.empty(t.shape, dtype=t.dtype, pin_memory=pin) for t in lp_dev)
                for host, dev_t in zip(lp, lp_dev):
                    host.copy_(dev_t, non_blocking=True)
        out = torch.empty(B, dtype=torch.int32, pin_memory=self.device.type == "cuda")
        out.copy_(tokens, non_blocking=True)
        self._feed_tokens[:B].copy_(tokens, non_blocking=True)  # the next step may read them on the device
        if self.device.type == "cuda":
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self._step_events.append((t_start, ev, plan.is_pure_decode))
        else:
            ev = None
        self._pending.append((plan, out, (ev, lp)))

    def collect(self):
        """Tokens of the oldest launched step."""
        plan, out, extra = self._pending.popleft()
        if out is None:
            return [], None
        ev, lp = extra
        if ev is not None:
            ev.synchronize()
        toks = out.tolist()
        logprobs = None
        if lp is not None:
            topv, topi, chosen = (t.tolist() for t in lp)
            logprobs = [{"top": [(i, v) for i, v in zip(topi[r], topv[r]) if i >= 0], "chosen": chosen[r]}
                        for r in range(len(toks))]
        return toks, logprobs

    def _upload_sampling(self, plan: StepPlan) -> dict:
        """The step's sampling arrays (``pack_sampling``) in one host-to-device copy
        from a pinned staging buffer; returns device views by name."""
        if self.device.type != "cuda":
            buf, layout = pack_sampling(plan)
            dev = torch.from_numpy(buf)
        else:
            i = self._samp_idx
            self._samp_idx ^= 1
            buf, layout = pack_sampling(plan, self._samp_pinned_np[i])
            n = buf.size
            if buf.base is None or n > self._samp_pinned[i].numel():  # grew past the staging buffer
                self._samp_pinned[i] = torch.empty(max(2 * n, 1024), dtype=torch.int32, pin_memory=True)
                self._samp_pinned_np[i] = self._samp_pinned[i].numpy()
                self._samp_pinned_np[i][:n] = buf
            if n > self._samp_dev.numel():
                self._samp_dev = torch.empty(max(2 * n, 1024), dtype=torch.int32, device=self.device)
            dev = self._samp_dev
            dev[:n].copy_(self._samp_pinned[i][:n], non_blocking=True)
            self.h2d_bytes += 4 * n
        views = {}
        for name, (o, n, dt) in layout.items():
            v = dev[o:o + n]
            views[name] = v.view(torch.float32) if dt == np.float32 else v.view(torch.int64) if dt == np.int64 else v
        if "allow" in views:
            views["allow"] = views["allow"].view(plan.grammar_rows.size, -1)
        return views

    def _sample(self, plan: StepPlan, logits: torch.Tensor):
        """Penalties, then ONE sampler kernel for every row (greedy, filtered and guided
        rows alike) that also writes the log-probabilities a row asked for.  Returns
        (tokens [B] int32, (top_v, top_i, chosen) device tensors or None)."""
        v = self._upload_sampling(plan)
        if plan.pen_rows is not None:
            ops.apply_penalties(logits, v["pen_rows"], v["pen_ids"], v["pen_counts"], v["presence"],
                                v["frequency"], v["repetition"])
        if plan.all_greedy and plan.grammar_rows is None and not plan.logprobs_k:
            return ops.argmax(logits), None
        B = plan.num_rows
        lp = None
        if plan.logprobs_k:
            k = plan.logprobs_k
            lp = (k, torch.empty(B, k, dtype=torch.float32, device=logits.device),
                  torch.empty(B, k, dtype=torch.int32, device=logits.device),
                  torch.empty(B, dtype=torch.float32, device=logits.device))
        seeds = v.get("seeds")
        if seeds is None:
            seeds = torch.zeros(B, dtype=torch.int64, device=logits.device)
        tokens = ops.sample(logits, v["temperature"], v.get("top_k"), v.get("top_p"), v.get("min_p"), seeds,
                            v.get("offsets"), allow=v.get("allow"), allow_row=v.get("allow_row"), logprobs=lp)
        return tokens, (lp[1:] if lp else None)

    # ----------------------------------------------------------- offload
    def offload_put(self, block_id: int) -> int:
        from b200moe.engine.kv_offload import HostBlockPool
        if self.offloader is None:
            self.offloader = HostBlockPool(self.config.kv_offload_host_blocks, self.kv, self.device)
        return self.offloader.put(block_id)

    def offload_get(self, slot: int, block_id: int):
        self.offloader.get(slot, block_id)

    def offload_release(self, slot: int):
        self.offloader.release(slot)

    # ----------------------------------------------------------- timing
    # ----------------------------------------------- int8 channel calibration
    def kv_calibrate_begin(self):
        """int8 channel mode: collect per-channel max |x| and sum |x| of every K / V the
        eager steps store (graph-replayed decode steps are not counted, as in the
        reference, whose hooks see prefill forwards only)."""
        if self.kv.int8_mode != "channel":
            raise RuntimeError("KV calibration needs kv_cache_dtype='int8' with kv_int8_mode='channel'")
        self.kv.calibrate_begin()
        self._calib_tokens = 0

    def kv_calibrate_freeze(self) -> int:
        """Freeze store / read scales and the outlier dims; returns the number of outlier dims."""
        if self._calib_tokens is None:
            raise RuntimeError("kv_calibrate_freeze without kv_calibrate_begin")
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        n = self.kv.calibrate_freeze(self._calib_tokens)
        self._calib_tokens = None
        return n

    def reset_step_timing(self):
        self._step_events.clear()
        ops.reset_launch_count()
        if self.model.ep is not None and self.model.ep.p2p is not None:
            self.model.ep.p2p.wait_stats(reset=True)

    def parallel_report(self) -> dict:
        """Which expert-parallel path and decode mode this rank runs, and (fused path)
        the device time its kernels waited on each peer since the last reset."""
        ep = self.model.ep
        rep = {"ep_backend": None if ep is None else ep.backend, "decode_graphs": sorted(self.graphs),
               "attention_parallel": "tp" if self.attn_tp > 1 else "dp",
               "tp_fused": self.model.tp_comm is not None}
        if ep is not None and ep.p2p is not None:
            torch.cuda.synchronize(self.device)
            rep["ep_wait"] = ep.p2p.wait_stats(reset=False)
        return rep

    def step_device_ms(self) -> float:
        """Sum of device time (upload start -> sampled ids ready) of the steps
        since the last reset."""
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        return float(sum(a.elapsed_time(b) for a, b, _ in self._step_events))

    def step_device_split(self) -> dict:
        """Device milliseconds and step counts of pure-decode steps and of steps
        that carry prefill rows, since the last reset."""
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        out = {"decode_ms": 0.0, "decode_steps": 0, "prefill_ms": 0.0, "prefill_steps": 0}
        for a, b, decode in self._step_events:
            k = "decode" if decode else "prefill"
            out[k + "_ms"] += a.elapsed_time(b)
            out[k + "_steps"] += 1
        return out

    def launch_count(self) -> int:
        return ops.launch_count()

    # -------------------------------------------------------------- misc
    def warmup(self):
        """One max-size prefill through the eager path (allocator + kernel first use)."""
        bs = self.block_size
        seq_len = min(self.max_tokens, self.config.max_model_len)
        nblk = -(-seq_len // bs)
        if nblk > self.config.num_kvcache_blocks:
            return
        pos = np.arange(seq_len, dtype=np.int32)
        tables = np.zeros((1, self.max_blocks), np.int32)
        tables[0, :nblk] = np.arange(nblk)
        plan = StepPlan(np.zeros(seq_len, np.int32), pos, pos.copy(), np.array([0, seq_len], np.int32),
                        np.array([seq_len], np.int32), tables, 0, seq_len, seq_len, np.zeros(1, np.int32),
                        np.zeros(1, np.float32))
        self.run(plan)

    def check_status(self):
        if self.device.type == "cuda":
            ops.check_status(self.device)

    # ------------------------------------------------------------ profiling
    def set_profiling(self, enabled: bool):
        """Start or stop the device-timed ranges on this rank (the model's
        per-segment ranges run on eager steps; graph replays time as one range)."""
        if enabled:
            self.profiler.start()
        else:
            self.profiler.stop()
        self.model.profiler = self.profiler if enabled else None

    def start_profiling(self):
        self.set_profiling(True)

    def stop_profiling(self):
        self.set_profiling(False)

    # ------------------------------------------- reference-compatible reports
    def call(self, method: str, *args):
        """Run ``method`` on every rank, returning this rank's result (the
        reference's ``model_runner.call``); without worker ranks, only here."""
        ex = getattr(self, "_executor", None)
        return ex.call(method, *args) if ex is not None else getattr(self, method)(*args)

    def memory_report(self) -> dict:
        gib = 2 ** 30
        cuda = self.device.type == "cuda"
        get = (lambda fn: fn(self.device) / gib) if cuda else (lambda fn: None)
        return {"rank": self.rank, "allocated_gib": get(torch.cuda.memory_allocated),
                "reserved_gib": get(torch.cuda.memory_reserved), "peak_gib": get(torch.cuda.max_memory_allocated)}

    def graph_report(self) -> dict:
        return {"rank": self.rank, "enabled": bool(self.graphs), "buckets": sorted(self.graphs),
                "kernels_per_replay": dict(self._graph_kernels), "memory": self.memory_report()}

    def set_enforce_eager(self, enabled: bool):
        self.set_cuda_graphs(not enabled)

    def warmup_model(self):
        self.warmup()

    def profile_snapshot(self, reset: bool = True) -> dict:
        """This rank's per-range and per-layer p50 / p95 (one device sync)."""
        out = self.profiler.snapshot(reset)
        out["rank"] = self.rank
        return out

    def exit(self):
        self.graphs.clear()
        self.graph_pool = None
        ep = getattr(getattr(self, "model", None), "ep", None)
        if ep is not None and getattr(ep, "p2p", None) is not None:
            ep.p2p.close()  # collective: every rank reaches exit together
            ep.p2p = None
        tp = getattr(getattr(self, "model", None), "tp_comm", None)
        if tp is not None:
            tp.close()  # collective, like the expert-parallel buffers
            self.model.tp_comm = None
        for attr in ("model", "kv"):
            if hasattr(self, attr):
                delattr(self, attr)
        gc.collect()
        if self.device.type == "cuda":
            torch.cuda.empty_cache()
        if self.world_size > 1:
            import torch.distributed as dist
            if dist.is_initialized():
                dist.destroy_process_group()
