"""Qwen3-MoE (and dense Qwen3) forward pass over the paged KV pool.

One decoder layer, CUDA path (every op a native sm_100a kernel):

    x   = rmsnorm(residual)                        (fused with the previous combine)
    qkv = gemm_tc(x, Wqkv e4m3)                    tcgen05, block-scaled
    q   = qknorm_rope_kvstore(qkv)                 k/v written to the paged pool
    o   = paged_{decode,prefill}_attn(q)
    x   = add_rmsnorm(gemm_tc(o, Wo e4m3), residual)
    moe: router gemm (bf16) -> router_topk -> permute -> gate_up+SiLU gemm
         -> down gemm (weighted scatter to the top-k slots)
    x   = moe_combine_add_rmsnorm(slots, residual) (next layer's input norm)

The CPU path runs the same math in fp32 torch ops (weights dequantised on the
fly) and is the oracle for the kernels.  Expert parallelism plugs in through
``self.ep`` (b200moe/parallel/ep.py): local tokens are dispatched to the ranks
that own their experts, computed there, and the weighted rows come back to
their (token, k) slots; the combine stays a fixed-order local sum.

Reference: nanovllm/models/qwen3_moe.py:69-490 and nanovllm/models/qwen3.py:14-216.
"""
from __future__ import annotations

from contextlib import nullcontext
from dataclasses import dataclass

import os

import torch
import torch.distributed as dist
from torch import nn

from b200moe import ops
from b200moe.config import ModelArgs
from b200moe.engine.kv_cache import KVPool


@dataclass
class StepInputs:
    """Device-side description of one forward step (rows = sequences).

    Decode rows (one query token) come first, then prefill rows.
    """
    input_ids: torch.Tensor        # int32 [T]
    positions: torch.Tensor        # int32 [T]
    slot_mapping: torch.Tensor     # int32 [T]
    cu_seqlens_q: torch.Tensor     # int32 [B + 1]
    seq_lens: torch.Tensor         # int32 [B] keys after this step
    block_tables: torch.Tensor     # int32 [B, max_blocks]
    logits_indices: torch.Tensor   # int32 [B] token index whose logits are sampled
    num_decode: int                # rows [0, num_decode) are single-token decode rows
    max_q_len: int                 # over prefill rows
    max_seq_len: int               # over all rows (decode split sizing)
    num_rows: int
    prefill_cu: torch.Tensor | None = None  # cu_seqlens of the prefill rows, rebased to 0
    feed_src: torch.Tensor | None = None    # int32 [T]: >= 0 -> the id is feed_tokens[feed_src[t]]
    feed_tokens: torch.Tensor | None = None  # previous step's sampled tokens (device)

    @property
    def num_tokens(self) -> int:
        return self.input_ids.shape[0]


def _param(t: torch.Tensor) -> nn.Parameter:
    return nn.Parameter(t, requires_grad=False)


class Qwen3MoeLayer(nn.Module):

    def __init__(self, args: ModelArgs, layer_id: int, num_local_experts: int, dtype, device, quant: bool,
                 nq: int | None = None, nkv: int | None = None):
        super().__init__()
        H, D = args.hidden_size, args.head_dim
        # nq / nkv: this rank's query / KV heads (all of them unless attention is tensor-parallel)
        nq = args.num_attention_heads if nq is None else nq
        nkv = args.num_key_value_heads if nkv is None else nkv
        self.layer_id = layer_id
        self.is_moe = args.is_moe_layer(layer_id)
        wdt = torch.float8_e4m3fn if quant else dtype
        nqkv = (nq + 2 * nkv) * D

        def w(*shape):
            return _param(torch.empty(*shape, dtype=wdt, device=device))

        def s(*shape):
            if not quant:
                return None
            *lead, n, k = shape
            return _param(torch.empty(*lead, n // 128, k // 128, dtype=torch.float32, device=device))

        self.input_layernorm = _param(torch.ones(H, dtype=dtype, device=device))
        self.post_attention_layernorm = _param(torch.ones(H, dtype=dtype, device=device))
        self.q_norm = _param(torch.ones(D, dtype=dtype, device=device))
        self.k_norm = _param(torch.ones(D, dtype=dtype, device=device))
        self.qkv_weight, self.qkv_scale = w(nqkv, H), s(nqkv, H)
        self.o_weight, self.o_scale = w(H, nq * D), s(H, nq * D)
        if self.is_moe:
            E, I = num_local_experts, args.moe_intermediate_size
            e_pad = -(-args.num_experts // 128) * 128
            self.router = _param(torch.zeros(e_pad, H, dtype=dtype, device=device))
        else:
            E, I = 1, args.intermediate_size
            self.router = None
        self.w13, self.s13 = w(E, 2 * I, H), s(E, 2 * I, H)
        self.w2, self.s2 = w(E, H, I), s(E, H, I)


class Qwen3MoeForCausalLM(nn.Module):

    def __init__(self, args: ModelArgs, device, dtype=None, ep_rank: int = 0, ep_size: int = 1,
                 expert_ids: list[int] | None = None, attn_tp: int = 1, attn_rank: int = 0):
        super().__init__()
        self.args = args
        # Tensor-parallel attention: this rank holds query heads
        # [q_head0, q_head0 + nq_local) and KV heads [kv_head0, kv_head0 + nkv_local)
        # (a KV head is replicated when there are more ranks than KV heads); the
        # O projection's partial sums and the local experts' outputs are
        # all-reduced over the ranks, which all see the same tokens.
        nq, nkv = args.num_attention_heads, args.num_key_value_heads
        if nq % attn_tp or (nkv % attn_tp and attn_tp % nkv):
            raise ValueError("tensor-parallel attention needs heads % tp == 0 and kv heads dividing or divisible by tp")
        self.attn_tp, self.attn_rank = attn_tp, attn_rank
        self.nq_local = nq // attn_tp
        self.nkv_local = max(1, nkv // attn_tp)
        self.q_head0 = attn_rank * self.nq_local
        self.kv_head0 = self.q_head0 // (nq // nkv)
        self.device = torch.device(device)
        self.dtype = dtype or (torch.bfloat16 if self.device.type == "cuda" else args.dtype)
        self.quant = args.quant_block is not None
        if self.quant and tuple(args.quant_block) != (128, 128):
            raise ValueError("only 128x128 fp8 weight blocks are supported")
        self.ep_rank, self.ep_size = ep_rank, ep_size
        E = args.num_experts
        self.num_local_experts = E // ep_size if args.is_moe else 0
        self.expert_ids = list(expert_ids) if expert_ids is not None else list(
            range(ep_rank * self.num_local_experts, (ep_rank + 1) * self.num_local_experts))
        H, V = args.hidden_size, args.vocab_size
        self.embed_tokens = _param(torch.empty(V, H, dtype=self.dtype, device=self.device))
        self.norm = _param(torch.ones(H, dtype=self.dtype, device=self.device))
        self.lm_head = self.embed_tokens if args.tie_word_embeddings else _param(
            torch.empty(V, H, dtype=self.dtype, device=self.device))
        self.layers = nn.ModuleList([
            Qwen3MoeLayer(args, l, self.num_local_experts, self.dtype, self.device, self.quant,
                          self.nq_local, self.nkv_local)
            for l in range(args.num_hidden_layers)])
        self.cos_sin = ops.rope_cos_sin(args.head_dim, args.max_position_embeddings, args.rope_theta, self.device)
        self.scale = args.head_dim ** -0.5
        self.ep = None          # expert-parallel communicator (multi-rank)
        self.tp_comm = None     # tensor-parallel attention: fused peer-memory sums (parallel/tp.py)
        self._tp_fused = False
        self.moe_backend = "fused"
        self.attention_backend = "paged"  # or "sdpa": per-sequence PyTorch attention (A/B, equivalence gate)
        self.profiler = None
        self._ws: dict = {}
        self.weights_tiled = False  # e4m3 GEMM weights stored tile-major (tile_weights_)

    # The e4m3 matrices the tcgen05 GEMM streams (QKV, O, expert gate/up and down).
    _TILED = ("qkv_weight", "o_weight", "w13", "w2")

    @torch.no_grad()
    def tile_weights_(self) -> None:
        """Re-lay every e4m3 GEMM weight tile-major in place (ops.tile_fp8): each
        pipeline stage of the GEMM then reads one contiguous 8 KB block of HBM.
        Loaders and reference paths see the natural layout through
        ``untile_weights_`` / ``natural``."""
        if self.weights_tiled or not self.quant or not self.cuda:
            return
        for layer in self.layers:
            for name in self._TILED:
                w = getattr(layer, name)
                w.copy_(ops.tile_fp8(w))
        self.weights_tiled = True

    @torch.no_grad()
    def cache_bf16_experts_(self) -> int:
        """Keep a bf16 copy of every MoE layer's expert weights, dequantised once
        (the same kernel and bits as the per-step dequantisation), for the steps
        large enough to run bf16 expert GEMMs (``_bf16_experts``): those then skip
        the per-step dequantisation pass.  Decode keeps reading e4m3 (half the
        bytes).  Returns the bytes held."""
        held = 0
        if not (self.cuda and self.quant and self.args.is_moe):
            return 0
        for layer in self.layers:
            if not layer.is_moe or getattr(layer, "w13_bf16", None) is not None:
                continue
            w13 = torch.empty(tuple(layer.w13.shape), dtype=torch.bfloat16, device=layer.w13.device)
            w2 = torch.empty(tuple(layer.w2.shape), dtype=torch.bfloat16, device=layer.w2.device)
            ops.dequant_weights(layer.w13, layer.s13, w13, self.weights_tiled)
            ops.dequant_weights(layer.w2, layer.s2, w2, self.weights_tiled)
            layer.w13_bf16, layer.w2_bf16 = w13, w2
            held += (w13.numel() + w2.numel()) * 2
        return held

    def bf16_expert_bytes(self) -> int:
        """Bytes ``cache_bf16_experts_`` would hold."""
        if not (self.quant and self.args.is_moe):
            return 0
        return sum((l.w13.numel() + l.w2.numel()) * 2 for l in self.layers if l.is_moe)

    @torch.no_grad()
    def untile_weights_(self) -> None:
        if not self.weights_tiled:
            return
        for layer in self.layers:
            for name in self._TILED:
                w = getattr(layer, name)
                w.copy_(ops.untile_fp8(w))
        self.weights_tiled = False

    def natural(self, w: torch.Tensor) -> torch.Tensor:
        """``w`` (one of the tiled matrices or a leading-index slice of one) in row-major layout."""
        return ops.untile_fp8(w) if self.weights_tiled else w

    def qkv_row_ranges(self) -> list[tuple[int, int]]:
        """Rows of the full [q | k | v] projection held by this rank (q, k, v order)."""
        a = self.args
        D, nq, nkv = a.head_dim, a.num_attention_heads, a.num_key_value_heads
        return [(self.q_head0 * D, (self.q_head0 + self.nq_local) * D),
                ((nq + self.kv_head0) * D, (nq + self.kv_head0 + self.nkv_local) * D),
                ((nq + nkv + self.kv_head0) * D, (nq + nkv + self.kv_head0 + self.nkv_local) * D)]

    def o_col_range(self) -> tuple[int, int]:
        """Input columns of the full O projection held by this rank."""
        D = self.args.head_dim
        return self.q_head0 * D, (self.q_head0 + self.nq_local) * D

    @property
    def cuda(self) -> bool:  # type: ignore[override]
        return self.device.type == "cuda"

    # ---------------------------------------------------------------- utils
    def _buf(self, name, shape, dtype):
        """Grow-only scratch buffers (stable addresses inside CUDA graphs once sized)."""
        n = 1
        for s in shape:
            n *= s
        t = self._ws.get((name, dtype))
        if t is None or t.numel() < n:
            t = torch.empty(max(n, 1), dtype=dtype, device=self.device)
            self._ws[(name, dtype)] = t
        return t[:n].view(*shape)

    def reserve_workspace(self, max_tokens: int, max_rows: int, max_splits: int):
        """Size every scratch buffer for the largest step up front."""
        a = self.args
        H, D, nq, nkv = a.hidden_size, a.head_dim, self.nq_local, self.nkv_local
        k = max(1, a.num_experts_per_tok)
        rows = max_tokens * k * max(1, self.ep_size)
        for name, shape, dt in (
                ("h", (max_tokens, H), self.dtype), ("x", (max_tokens, H), self.dtype),
                ("qkv", (max_tokens, (nq + 2 * nkv) * D), self.dtype), ("q", (max_tokens, nq, D), self.dtype),
                ("attn", (max_tokens, nq, D), self.dtype), ("o", (max_tokens, H), self.dtype),
                ("part_o", (max_rows * nq * max_splits, D), torch.float32),
                ("part_m", (max_rows * nq * max_splits,), torch.float32),
                ("part_l", (max_rows * nq * max_splits,), torch.float32)):
            self._buf(name, shape, dt)
        I = max(a.moe_intermediate_size, a.intermediate_size)
        if a.is_moe:
            self._buf("rlogits", (max_tokens, -(-a.num_experts // 128) * 128), torch.float32)
            self._buf("x_perm", (rows, H), self.dtype)
            self._buf("slots", (max_tokens * k, H), self.dtype)
            self._buf("slot_of_row", (rows,), torch.int32)
            self._buf("ids", (max_tokens * k,), torch.int32)
            self._buf("topw", (max_tokens * k,), torch.float32)
        self._buf("h_perm", (max(rows, max_tokens), I), self.dtype)
        if self._bf16_experts(rows) and self.layers and getattr(self.layers[0], "w13_bf16", None) is None:
            l0 = self.layers[0]
            self._buf("w13_bf16", tuple(l0.w13.shape), torch.bfloat16)
            self._buf("w2_bf16", tuple(l0.w2.shape), torch.bfloat16)

    # Routed rows per expert from which a step dequantises the layer's expert
    # weights to bf16 once and runs the bf16 grouped GEMMs: below it the e4m3
    # GEMMs (dequantising per tile) win; above it every expert's weights are
    # re-dequantised for many token tiles (B200MOE_BF16_EXPERT_ROWS, 0 = never).
    BF16_EXPERT_ROWS = int(os.environ.get("B200MOE_BF16_EXPERT_ROWS", "512"))

    def _bf16_experts(self, rows: int) -> bool:
        E = max(1, self.num_local_experts)
        return (self.cuda and self.quant and self.args.is_moe and self.BF16_EXPERT_ROWS > 0
                and rows >= self.BF16_EXPERT_ROWS * E)

    def _range(self, name: str):
        return nullcontext() if self.profiler is None else self.profiler.range(name)

    # -------------------------------------------------------------- forward
    @torch.inference_mode()
    def forward(self, inp: StepInputs, kv: KVPool) -> torch.Tensor:
        """Returns the final hidden states of the ``logits_indices`` rows."""
        a = self.args
        T = inp.num_tokens
        H = a.hidden_size
        eps = a.rms_norm_eps
        cuda = self.cuda
        feed = (inp.feed_src, inp.feed_tokens) if inp.feed_src is not None else None
        residual = ops.embed(inp.input_ids, self.embed_tokens, out=self._buf("h", (T, H), self.dtype) if cuda else None,
                             feed=feed)
        x = ops.rmsnorm(residual, self.layers[0].input_layernorm, eps,
                        out=self._buf("x", (T, H), self.dtype) if cuda else None)
        # tensor-parallel attention: decode-size batches sum the ranks' partials over peer memory
        self._tp_fused = self.attn_tp > 1 and self.tp_comm is not None and T <= self.tp_comm.max_tokens
        if self._tp_fused:
            self.tp_comm.begin_forward(len(self.layers) + sum(1 for ly in self.layers if ly.is_moe))
        for l, layer in enumerate(self.layers):
            attn = self._attention(layer, x, inp, kv.layer(l))
            xbuf = self._buf("x", (T, H), self.dtype) if cuda else None
            if self._tp_fused:
                with self._range("attn.o_proj_allreduce_norm"):
                    x = self.tp_comm.o_proj_add_norm(attn, layer.o_weight, layer.o_scale, residual,
                                                     layer.post_attention_layernorm, eps, xbuf, self.weights_tiled)
            elif self.attn_tp > 1:
                with self._range("attn.o_proj"):
                    o = ops.linear(attn, layer.o_weight, layer.o_scale,
                                   out=self._buf("o", (T, H), self.dtype) if cuda else None, tiled=self.weights_tiled)
                with self._range("attn.all_reduce"):
                    dist.all_reduce(o)  # row-parallel O projection: sum of the ranks' partial products
                x = ops.rmsnorm(o, layer.post_attention_layernorm, eps, residual=residual, out=xbuf)
            else:
                with self._range("attn.o_proj_add_norm"):
                    x = ops.linear_add_rmsnorm(attn, layer.o_weight, layer.o_scale, residual,
                                               layer.post_attention_layernorm, eps, out=xbuf,
                                               tiled=self.weights_tiled)
            nxt = self.layers[l + 1].input_layernorm if l + 1 < len(self.layers) else self.norm
            x = self._mlp(layer, x, residual, nxt, T)
        return x.index_select(0, inp.logits_indices.long())

    def compute_logits(self, h: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """fp32 logits [rows, vocab] (LM head on the tcgen05 GEMM, bf16 weights)."""
        return ops.linear(h, self.lm_head, None, out_dtype=torch.float32, out=out)

    def _attention(self, layer, x, inp: StepInputs, kvl):
        a = self.args
        T = inp.num_tokens
        nq, nkv, D = self.nq_local, self.nkv_local, a.head_dim
        cuda = self.cuda
        with self._range("attn.qkv_norm_rope_kvstore"):
            q = ops.qkv_norm_rope_kvstore(x, layer.qkv_weight, layer.qkv_scale, inp.positions, inp.slot_mapping,
                                          layer.q_norm, layer.k_norm, self.cos_sin, kvl, nq, nkv, D,
                                          a.rms_norm_eps,
                                          self._buf("qkv", (T, (nq + 2 * nkv) * D), self.dtype) if cuda else None,
                                          self._buf("q", (T, nq, D), self.dtype) if cuda else None,
                                          tiled=self.weights_tiled)
        out = self._buf("attn", (T, nq, D), self.dtype) if cuda else torch.empty(T, nq, D, dtype=q.dtype)
        nd = inp.num_decode
        with self._range("attn.core"):
            cu = inp.prefill_cu if inp.prefill_cu is not None else inp.cu_seqlens_q
            if cuda and self.attention_backend == "sdpa":
                if nd:
                    ops._attention_ref(q[:nd], kvl, inp.block_tables[:nd], inp.seq_lens[:nd],
                                       torch.arange(nd + 1, dtype=torch.int32), self.scale, out[:nd])
                if inp.num_rows > nd:
                    ops._attention_ref(q[nd:], kvl, inp.block_tables[nd:], inp.seq_lens[nd:], cu, self.scale,
                                       out[nd:])
            else:
                if nd:
                    split_len, nsplit = self.decode_splits(nd, inp.max_seq_len)
                    ws = None
                    if cuda:
                        ws = (self._buf("part_o", (nd * nq * nsplit, D), torch.float32),
                              self._buf("part_m", (nd * nq * nsplit,), torch.float32),
                              self._buf("part_l", (nd * nq * nsplit,), torch.float32))
                    ops.decode_attention(q[:nd], kvl, inp.block_tables[:nd], inp.seq_lens[:nd], self.scale,
                                         out[:nd], split_len, nsplit, ws)
                if inp.num_rows > nd:
                    ops.prefill_attention(q[nd:], kvl, cu, inp.seq_lens[nd:], inp.block_tables[nd:],
                                          inp.max_q_len, self.scale, out[nd:])
        return out.view(T, nq * D)  # the O projection is applied by the caller

    def decode_splits(self, rows: int, max_len: int) -> tuple[int, int]:
        """Keys per split and split count for flash-decoding: enough CTAs to
        cover the SMs a few times over, splits of at least 64 keys."""
        nkv = getattr(self, "nkv_local", self.args.num_key_value_heads)
        want = max(1, -(-4 * ops.NUM_SMS // max(1, rows * nkv)))
        split_len = max(64, -(-max(1, max_len) // want))
        split_len = -(-split_len // 64) * 64
        return split_len, max(1, -(-max(1, max_len) // split_len))

    # ------------------------------------------------------------------ MLP
    def _mlp(self, layer, x, residual, next_norm, T):
        a = self.args
        eps = a.rms_norm_eps
        if not layer.is_moe:
            return self._dense_mlp(layer, x, residual, next_norm, T)
        if self.attn_tp > 1:
            return self._moe_tp(layer, x, residual, next_norm, T)
        if not self.cuda or self.moe_backend == "loop":
            moe_out = self._moe_reference(layer, x)
            return ops.rmsnorm(moe_out, next_norm, eps, residual=residual,
                               out=self._buf("x", (T, a.hidden_size), self.dtype) if self.cuda else None)
        slots = self._moe_fused(layer, x, T)
        with self._range("moe.combine_norm"):
            # the combine kernel also clears the routing counters for the next layer
            counts = self._buf("counts", (2 * a.num_experts + 1,), torch.int32) if self.ep is None else None
            out = ops.moe_combine_add_rmsnorm(slots, a.num_experts_per_tok, residual, next_norm, eps,
                                              out=self._buf("x", (T, a.hidden_size), self.dtype), zero=counts,
                                              wait=self.ep.combine_wait() if self.ep is not None else None)
            self._counts_clear = counts is not None
            return out

    def route(self, layer, x, counts=None):
        """Router GEMM + top-k: (ids [T, k] int32, weights [T, k] fp32)."""
        a = self.args
        T = x.shape[0]
        k = a.num_experts_per_tok
        cuda = x.is_cuda
        ids = self._buf("ids", (T * k,), torch.int32).view(T, k) if cuda else torch.empty(T, k, dtype=torch.int32)
        w = self._buf("topw", (T * k,), torch.float32).view(T, k) if cuda else torch.empty(T, k)
        if cuda and a.num_experts <= 128 and layer.router.dtype == torch.bfloat16:
            ops.router_fused(x, layer.router, a.num_experts, k, a.norm_topk_prob, ids, w, counts)
            return ids, w
        logits = ops.linear(x, layer.router, None, out_dtype=torch.float32,
                            out=self._buf("rlogits", (T, layer.router.shape[0]), torch.float32) if cuda else None)
        ops.router_topk(logits, a.num_experts, k, a.norm_topk_prob, ids, w, counts)
        return ids, w

    def _moe_reference(self, layer, x):
        """fp32 torch MoE: each local expert on its routed rows, fixed-order sum."""
        ids, w = self.route(layer, x)
        if self.ep is not None:
            return self.ep.moe_reference(self, layer, x, ids, w)
        return self.experts_reference(layer, x, ids, w).sum(dim=1).to(x.dtype)

    def experts_reference(self, layer, x, ids, w):
        """Weighted expert outputs per (token, k) slot [T, k, H] (fp32; bf16
        rounding points of the native path when x is bf16).  Slots whose
        expert is not local stay zero."""
        T, H = x.shape
        k = ids.shape[1]
        I = layer.w2.shape[-1]
        bf = x.dtype == torch.bfloat16
        slots = torch.zeros(T, k, H, dtype=torch.float32, device=x.device)
        for le, ge in enumerate(self.expert_ids):
            mask = ids == ge
            if not bool(mask.any()):
                continue
            t_idx, k_idx = mask.nonzero(as_tuple=True)
            w13 = ops.dequant_block_fp8(self.natural(layer.w13[le]), layer.s13[le]) if self.quant \
                else layer.w13[le].float()
            w2 = ops.dequant_block_fp8(self.natural(layer.w2[le]), layer.s2[le]) if self.quant else layer.w2[le].float()
            if bf:  # the native GEMM dequantises to bf16 before the MMA
                w13, w2 = w13.to(torch.bfloat16).float(), w2.to(torch.bfloat16).float()
            gu = x[t_idx].float() @ w13.t()
            h = torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]
            if bf:
                h = h.to(torch.bfloat16).float()
            y = (h @ w2.t()) * w[t_idx, k_idx].unsqueeze(1)
            slots[t_idx, k_idx] = y.to(torch.bfloat16).float() if bf else y
        return slots

    def _moe_fused(self, layer, x, T):
        a = self.args
        k = a.num_experts_per_tok
        H = a.hidden_size
        E = a.num_experts
        I = layer.w2.shape[-1]
        slots = self._buf("slots", (T * k, H), self.dtype)
        counts = self._buf("counts", (2 * E + 1,), torch.int32)
        with self._range("moe.router"):
            if self.ep is None and not getattr(self, "_counts_clear", False):
                counts.zero_()  # otherwise the previous layer's combine kernel cleared them
            self._counts_clear = False
            routed = self.ep.route_dispatch(self, layer, x) if self.ep is not None else None
            dispatched = routed is not None
            ids, w = routed if dispatched else self.route(layer, x, counts[:E] if self.ep is None else None)
        if self.ep is not None:
            with self._range("moe.ep"):
                return self.ep.moe_fused(self, layer, x, ids, w, slots, dispatched)
        rows = T * k
        with self._range("moe.permute"):
            x_perm = self._buf("x_perm", (rows, H), self.dtype)
            slot_of_row = self._buf("slot_of_row", (rows,), torch.int32)
            offsets = self._buf("offsets", (E + 1,), torch.int32)
            ops.moe_permute(x, ids, counts[:E], counts[E:2 * E], x_perm, slot_of_row, offsets)
        if self.profiler is not None:
            self.profiler.observe("moe.max_expert_rows", counts[:E].max())  # routing imbalance
        if self._bf16_experts(rows):
            # large prefill batch: bf16 GEMMs (no per-tile dequantisation) on the resident
            # bf16 copy (cache_bf16_experts_) or on a copy dequantised for this step
            w13, w2 = getattr(layer, "w13_bf16", None), getattr(layer, "w2_bf16", None)
            if w13 is None:
                w13 = self._buf("w13_bf16", tuple(layer.w13.shape), torch.bfloat16)
                w2 = self._buf("w2_bf16", tuple(layer.w2.shape), torch.bfloat16)
                with self._range("moe.dequant"):
                    ops.dequant_weights(layer.w13, layer.s13, w13, self.weights_tiled)
                    ops.dequant_weights(layer.w2, layer.s2, w2, self.weights_tiled)
            s13 = s2 = None
            tiled = False
        else:
            w13, s13, w2, s2, tiled = layer.w13, layer.s13, layer.w2, layer.s2, self.weights_tiled
        with self._range("moe.gate_up"):
            h_perm = self._buf("h_perm", (rows, I), self.dtype)
            ops.grouped_gate_up_silu(x_perm, w13, s13, counts[:E], offsets, h_perm, I, tiled=tiled)
        with self._range("moe.down"):
            ops.grouped_down_scatter(h_perm, w2, s2, counts[:E], offsets, slot_of_row,
                                     w.view(-1), slots, tiled=tiled)
        return slots

    def _moe_tp(self, layer, x, residual, next_norm, T):
        """Tensor-parallel attention mode: every rank holds all T tokens; it runs
        its own experts on the tokens routed to them, and the ranks' partial sums
        are all-reduced before the residual add (the reference's EP combine,
        nanovllm/models/qwen3_moe.py:414-418)."""
        a = self.args
        k, H, E, eps = a.num_experts_per_tok, a.hidden_size, a.num_experts, a.rms_norm_eps
        El = self.num_local_experts
        partial = self._buf("moe_partial", (T, H), self.dtype) if self.cuda else torch.zeros(T, H, dtype=x.dtype)
        if not self.cuda or self.moe_backend == "loop":
            ids, w = self.route(layer, x)
            partial.copy_(self.experts_reference(layer, x, ids, w).sum(1).to(partial.dtype))
        else:
            counts = self._buf("counts", (2 * E + 1,), torch.int32)
            counts.zero_()
            ids, w = self.route(layer, x, counts[:E])
            g2l = self._tp_maps()
            ids_l = g2l.index_select(0, ids.reshape(-1).long()).view(T, k)   # -1: another rank's expert
            counts_l = self._buf("counts_l", (2 * El,), torch.int32)
            counts_l[:El].copy_(counts[:E].index_select(0, self._expert_ids_dev))
            counts_l[El:].zero_()
            rows = T * k
            x_perm = self._buf("x_perm", (rows, H), self.dtype)
            slot_of_row = self._buf("slot_of_row", (rows,), torch.int32)
            offsets = self._buf("offsets", (El + 1,), torch.int32)
            ops.moe_permute(x, ids_l, counts_l[:El], counts_l[El:], x_perm, slot_of_row, offsets)
            I = layer.w2.shape[-1]
            h_perm = self._buf("h_perm", (rows, I), self.dtype)
            ops.grouped_gate_up_silu(x_perm, layer.w13, layer.s13, counts_l[:El], offsets, h_perm, I,
                                     tiled=self.weights_tiled)
            slots = self._buf("slots", (rows, H), self.dtype)
            slots.zero_()  # slots of other ranks' experts stay zero
            ops.grouped_down_scatter(h_perm, layer.w2, layer.s2, counts_l[:El], offsets, slot_of_row,
                                     w.view(-1), slots, tiled=self.weights_tiled)
            if self._tp_fused:
                with self._range("moe.allreduce_norm"):
                    return self.tp_comm.slots_add_norm(slots, k, residual, next_norm, eps,
                                                       self._buf("x", (T, H), self.dtype))
            # combine (fixed-order sum over k) into a zeroed residual: partial = sum_k slots
            partial.zero_()
            ops.moe_combine_add_rmsnorm(slots, k, partial, next_norm, eps,
                                        out=self._buf("moe_norm_scratch", (T, H), self.dtype))
        with self._range("moe.all_reduce"):
            dist.all_reduce(partial)
        return ops.rmsnorm(partial, next_norm, eps, residual=residual,
                           out=self._buf("x", (T, H), self.dtype) if self.cuda else None)

    def _tp_maps(self):
        g2l = getattr(self, "_g2l_dev", None)
        if g2l is None:
            E = self.args.num_experts
            m = torch.full((E,), -1, dtype=torch.int32)
            for le, ge in enumerate(self.expert_ids):
                m[ge] = le
            self._g2l_dev = g2l = m.to(self.device)
            self._expert_ids_dev = torch.tensor(self.expert_ids, dtype=torch.long, device=self.device)
        return g2l

    def _dense_mlp(self, layer, x, residual, next_norm, T):
        a = self.args
        eps = a.rms_norm_eps
        I = layer.w2.shape[-1]
        if not self.cuda:
            w13 = ops.dequant_block_fp8(layer.w13[0], layer.s13[0]) if self.quant else layer.w13[0].float()
            w2 = ops.dequant_block_fp8(layer.w2[0], layer.s2[0]) if self.quant else layer.w2[0].float()
            gu = x.float() @ w13.t()
            h = (torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]).to(x.dtype)
            y = (h.float() @ w2.t()).to(x.dtype)
            return ops.rmsnorm(y, next_norm, eps, residual=residual)
        h = self._buf("h_perm", (T, I), self.dtype)
        ops.grouped_gate_up_silu(x, layer.w13, layer.s13, ops.count_tensor(T, x.device), None, h, I,
                                 tiled=self.weights_tiled)
        y = ops.linear(h, layer.w2[0], layer.s2[0] if self.quant else None, tiled=self.weights_tiled,
                       out=self._buf("o", (T, a.hidden_size), self.dtype))
        return ops.rmsnorm(y, next_norm, eps, residual=residual, out=self._buf("x", (T, a.hidden_size), self.dtype))
