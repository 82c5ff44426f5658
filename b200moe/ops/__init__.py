"""Python entry points of the sm_100a kernels.

CUDA tensors always go to the native extension (``b200moe._C``); if it is
missing on a GPU the call raises, it never falls back to a slower path.  CPU
tensors take the plain-PyTorch fp32 definition of the same op, which is the
numerics oracle used by the tests and by the CPU engine.
"""
from __future__ import annotations

import math
import os

import torch

try:  # the in-tree build (python setup.py build_ext --inplace)
    from b200moe import _C  # type: ignore
    _IMPORT_ERROR = None
except Exception as exc:  # pragma: no cover - depends on the build
    _C = None
    _IMPORT_ERROR = exc

EPI_BF16, EPI_F32, EPI_SILU_PAIR, EPI_SCATTER = 0, 1, 2, 3
NUM_SMS = 148


_launches = [0]


def count_launches(n: int = 1):
    _launches[0] += n


def launch_count() -> int:
    """Native kernels launched by this process since the last reset."""
    return _launches[0]


def reset_launch_count():
    _launches[0] = 0


def native():
    if _C is None:
        raise RuntimeError(
            "b200moe native extension is not built (run `python setup.py build_ext --inplace`): "
            f"{_IMPORT_ERROR}")
    return _C


def native_available() -> bool:
    return _C is not None


_trace = [None]  # optional int64 buffer: GEMM pipeline trace of CTA 0 (profiling only)


def set_gemm_trace(buf: torch.Tensor | None):
    _trace[0] = buf


_status_cache: dict = {}
_count_cache: dict = {}


def status_word(device) -> torch.Tensor:
    """Per-device int32 status word that kernels set on a bounded-wait timeout."""
    key = torch.device(device)
    t = _status_cache.get(key)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=key)
        _status_cache[key] = t
    return t


def check_status(device) -> None:
    """Raise if a kernel on ``device`` recorded an error (reads one int: a sync)."""
    t = _status_cache.get(torch.device(device))
    if t is not None:
        v = int(t.item())
        if v != 0:
            t.zero_()
            raise RuntimeError(f"device kernel reported status {v} (bounded wait expired or bad input)")


def count_tensor(n: int, device) -> torch.Tensor:
    """Cached one-element int32 device tensor holding ``n`` (dense GEMM group count)."""
    key = (n, torch.device(device))
    t = _count_cache.get(key)
    if t is None:
        t = torch.tensor([n], dtype=torch.int32, device=device)
        _count_cache[key] = t
    return t


# --------------------------------------------------------------- references
def dequant_block_fp8(w: torch.Tensor, scale: torch.Tensor, block: int = 128) -> torch.Tensor:
    """fp32 value of a 128x128 block-scaled e4m3 weight ([..., N, K])."""
    wf = w.float()
    s = scale.float().repeat_interleave(block, dim=-2)[..., :wf.shape[-2], :]
    s = s.repeat_interleave(block, dim=-1)[..., :wf.shape[-1]]
    return wf * s


def dequant_block_fp8_bf16(w, scale, block=128):
    """The reference's load-time dequant: bf16(float(q) * scale) (loader.py:28-35)."""
    return dequant_block_fp8(w, scale, block).to(torch.bfloat16)


def pick_bn(rows: int, m_tiles: int, groups: int = 1, pair: bool = False, sms: int = NUM_SMS) -> int:
    """Token tile of the tcgen05 GEMM: the largest tile that still gives the
    persistent grid one work item per SM, and no larger than twice the rows a
    group is expected to hold."""
    per_group = max(1, math.ceil(rows / max(groups, 1)))
    choices = (16, 32, 64, 128) if pair else (16, 32, 64, 128, 256)
    best = choices[0]
    for bn in choices[1:]:
        if bn > 2 * per_group:
            break
        if groups * math.ceil(per_group / bn) * m_tiles < sms:
            break
        best = bn
    return best


def _dense_cost_us(rows: int, m_tiles: int, k_stages: int, bn: int, splits: int, sms: int, fp8: bool) -> float:
    """Rough time model of the persistent GEMM: waves of work items, each a
    run of K stages costing the slower of weight-tile preparation (fp8
    dequantisation or the bf16 tile load) and the MMA, plus its epilogue, plus
    the partial-sum traffic of split-K.  Constants are B200 measurements of
    this kernel, rounded."""
    n_tiles = math.ceil(rows / bn)
    items = m_tiles * n_tiles * splits
    waves = math.ceil(items / sms)
    per = math.ceil(k_stages / splits)
    stage = max(0.15 if fp8 else 0.08, 0.0011 * bn) + 0.02
    t = waves * (per * stage + 0.3 + 0.004 * bn) + 1.0
    if splits > 1:
        t += 2.0 + splits * rows * m_tiles * 128 * 4 * 2 / 5e6
    return t


def plan_dense(rows: int, m_tiles: int, k_stages: int, sms: int = NUM_SMS, fp8: bool = True,
               max_splits: int = 1 << 30) -> tuple[int, int]:
    """(token tile, K splits) of a single-group GEMM, the cheapest under
    ``_dense_cost_us``.  Decode-size token counts give too few output tiles to
    fill the grid (o_proj at 256 tokens is 16 weight tiles): a larger token
    tile dequantises each weight tile fewer times, and splitting K spreads the
    stages over the SMs; the fp32 partials are summed by a small kernel."""
    best, best_t = (pick_bn(rows, m_tiles, sms=sms), 1), float("inf")
    for bn in (16, 32, 64, 128, 256):
        if bn > 16 and bn >= 2 * rows:
            break
        # e4m3 tiles of up to 128 tokens run 128-wide K stages (two 64-wide blocks)
        ks = k_stages // 2 if fp8 and bn <= 128 else k_stages
        for splits in range(1, max(1, min(ks // 2, max_splits)) + 1):
            per = math.ceil(ks / splits)
            if math.ceil(ks / per) != splits:
                continue  # would leave a split empty
            t = _dense_cost_us(rows, m_tiles, k_stages, bn, splits, sms, fp8)
            if t < best_t:
                best, best_t = (bn, splits), t
    return best


# Token count from which an e4m3 dense GEMM dequantises its weight once and runs
# in bf16 (B200MOE_BF16_DENSE_ROWS, 0 = never).
BF16_DENSE_ROWS = int(os.environ.get("B200MOE_BF16_DENSE_ROWS", "2048"))
_scratch_bufs: dict = {}


def _scratch(name: str, numel: int, dtype, device) -> torch.Tensor:
    """Grow-only per-device scratch (eager prefill paths only, never inside a graph capture)."""
    key = (name, dtype, torch.device(device))
    t = _scratch_bufs.get(key)
    if t is None or t.numel() < numel:
        t = torch.empty(numel, dtype=dtype, device=device)
        _scratch_bufs[key] = t
    return t[:numel]


# ------------------------------------------------------- weight layout
def _swizzle64_index(device) -> torch.Tensor:
    # chunk u (16 bytes) of row r of a [128][64 B] block sits at chunk u ^ ((r >> 1) & 3)
    r = torch.arange(128, device=device).view(128, 1)
    u = torch.arange(4, device=device).view(1, 4)
    return (u ^ ((r >> 1) & 3)).view(128, 4, 1).expand(128, 4, 16)


def tile_fp8(w: torch.Tensor) -> torch.Tensor:
    """[..., N, K] e4m3 -> the same shape holding the bytes tile-major:
    [..., N / 128, K / 64, 128, 64] with the four 16-byte chunks of each 64-byte
    row in 64-byte-swizzle order (chunk u of row r at u ^ ((r >> 1) & 3)).  One
    GEMM pipeline stage (128 rows x 64 K) is then one contiguous 8 KB block that a
    single bulk copy brings into shared memory already in the layout the
    dequantisers read without bank conflicts."""
    *lead, n, k = w.shape
    if n % 128 or k % 64:
        raise ValueError("tile_fp8 needs N % 128 == 0 and K % 64 == 0")
    b = w.view(torch.uint8).reshape(*lead, n // 128, 128, k // 64, 64).transpose(-3, -2).contiguous()
    b = b.view(-1, 128, 4, 16)
    idx = _swizzle64_index(w.device).unsqueeze(0).expand(b.shape[0], 128, 4, 16)
    out = torch.empty_like(b).scatter_(2, idx, b)
    return out.view(w.shape).view(w.dtype)


def untile_fp8(w: torch.Tensor) -> torch.Tensor:
    """Inverse of ``tile_fp8``."""
    *lead, n, k = w.shape
    b = w.view(torch.uint8).reshape(-1, 128, 4, 16)
    idx = _swizzle64_index(w.device).unsqueeze(0).expand(b.shape[0], 128, 4, 16)
    b = torch.gather(b, 2, idx)
    b = b.view(*lead, n // 128, k // 64, 128, 64).transpose(-3, -2).contiguous()
    return b.view(w.shape).view(w.dtype)


# --------------------------------------------------------------------- GEMM
def linear(x: torch.Tensor, weight: torch.Tensor, scale: torch.Tensor | None, out_dtype=torch.bfloat16,
           out: torch.Tensor | None = None, tiled: bool = False) -> torch.Tensor:
    """y = x @ W^T with W either block-scaled e4m3 (+ scale) or bf16/fp32.
    ``tiled``: the e4m3 weight is stored tile-major (``tile_fp8``)."""
    T = x.shape[0]
    N = weight.shape[0]
    if not x.is_cuda:
        if tiled:
            weight = untile_fp8(weight)
        w = dequant_block_fp8(weight, scale) if scale is not None else weight.float()
        y = x.float() @ w.t()
        return y.to(out_dtype) if out is None else out.copy_(y)
    C = native()
    if out is None:
        out = torch.empty(T, N, dtype=out_dtype, device=x.device)
    if T == 0:
        return out
    if scale is not None and T >= BF16_DENSE_ROWS > 0 and weight.dim() == 2:
        # prefill-size batch: one dequantisation of the (small) weight into a scratch,
        # then the bf16 GEMM instead of dequantising every weight tile per token tile
        wb = _scratch("dense_bf16", weight.numel(), torch.bfloat16, x.device).view(weight.shape)
        dequant_weights(weight, scale, wb, tiled)
        weight, scale, tiled = wb, None, False
    m_tiles = N // 128
    bn, splits = plan_dense(T, m_tiles, x.shape[1] // 64, fp8=scale is not None)
    if splits > 1:
        part = torch.empty(splits * T, N, dtype=torch.float32, device=x.device)
        C.gemm(weight, scale, x, count_tensor(T, x.device), None, part, bn, EPI_F32, m_tiles,
               0, 0, None, None, status_word(x.device), _trace[0], splits, T * N, tiled, [])
        C.splitk_reduce(part, splits, out)
        count_launches(2)
        return out
    epi = EPI_F32 if out.dtype == torch.float32 else EPI_BF16
    C.gemm(weight, scale, x, count_tensor(T, x.device), None, out, bn, epi, m_tiles,
           0, 0, None, None, status_word(x.device), _trace[0], 1, 0, tiled, [])
    count_launches()
    return out


def linear_add_rmsnorm(x, weight, scale, residual, norm_w, eps, out, tiled: bool = False):
    """residual += bf16(x @ W^T); return rmsnorm(residual) * norm_w.  When the
    planner splits K, the fp32 partial sums go straight into the norm kernel
    (no separate reduce launch, no bf16 round trip through memory)."""
    T, N = x.shape[0], weight.shape[0]
    if not x.is_cuda or T == 0:
        return rmsnorm(linear(x, weight, scale, tiled=tiled), norm_w, eps, residual=residual, out=out)
    m_tiles = N // 128
    bn, splits = plan_dense(T, m_tiles, x.shape[1] // 64, fp8=scale is not None)
    if splits == 1:
        return rmsnorm(linear(x, weight, scale, tiled=tiled), norm_w, eps, residual=residual, out=out)
    C = native()
    part = torch.empty(splits * T, N, dtype=torch.float32, device=x.device)
    C.gemm(weight, scale, x, count_tensor(T, x.device), None, part, bn, EPI_F32, m_tiles,
           0, 0, None, None, status_word(x.device), _trace[0], splits, T * N, tiled, [])
    C.rmsnorm_partials(part, splits, residual, norm_w, out, eps)
    count_launches(2)
    return out


def grouped_gate_up_silu(x_perm, w13, s13, counts, offsets, out, inter: int, bn: int | None = None,
                         tiled: bool = False):
    """out[r] = silu(x_perm[r] @ Wg_e^T) * (x_perm[r] @ Wu_e^T) for the rows of expert e."""
    C = native()
    rows = x_perm.shape[0]
    m_tiles = inter // 128
    bn = bn or pick_bn(rows, m_tiles, groups=w13.shape[0], pair=True)
    C.gemm(w13, s13, x_perm, counts, offsets, out, bn, EPI_SILU_PAIR, m_tiles, inter, 0, None, None,
           status_word(x_perm.device), _trace[0], 1, 0, tiled, [])
    count_launches()
    return out


def grouped_down_scatter(h_perm, w2, s2, counts, offsets, slot_of_row, slot_weight, slots_out,
                         bn: int | None = None, tiled: bool = False):
    """slots_out[slot_of_row[r]] = (h_perm[r] @ Wd_e^T) * slot_weight[slot] for the rows of expert e."""
    C = native()
    rows = h_perm.shape[0]
    m_tiles = w2.shape[1] // 128
    bn = bn or pick_bn(rows, m_tiles, groups=w2.shape[0])
    C.gemm(w2, s2, h_perm, counts, offsets, slots_out, bn, EPI_SCATTER, m_tiles, 0, 0, slot_of_row, slot_weight,
           status_word(h_perm.device), _trace[0], 1, 0, tiled, [])
    count_launches()
    return slots_out


def dequant_weights(q: torch.Tensor, scale: torch.Tensor, out: torch.Tensor, tiled: bool = False) -> torch.Tensor:
    """bf16(float(q) * block scale) of an e4m3 weight stack [..., N, K] into ``out``
    (row-major bf16); ``tiled``: q is stored tile-major (``tile_fp8``)."""
    if not q.is_cuda:
        w = untile_fp8(q) if tiled else q
        lead = w.shape[:-2]
        flat_w, flat_s = w.reshape(-1, *w.shape[-2:]), scale.reshape(-1, *scale.shape[-2:])
        res = torch.stack([dequant_block_fp8(flat_w[i], flat_s[i]) for i in range(flat_w.shape[0])])
        return out.copy_(res.view(*lead, *w.shape[-2:]).to(out.dtype))
    native().dequant_weights(q, scale, out, tiled)
    count_launches()
    return out


# -------------------------------------------------------------- fused ops
def embed(ids: torch.Tensor, table: torch.Tensor, out: torch.Tensor | None = None,
          feed: tuple[torch.Tensor, torch.Tensor] | None = None) -> torch.Tensor:
    """Embedding rows of ``ids``; ``feed = (src, tokens)``: token t takes its id
    from ``tokens[src[t]]`` where ``src[t] >= 0`` (the previous step's sampled
    tokens, still on the device)."""
    if not ids.is_cuda:
        if feed is not None:
            src, toks = feed
            src = src[:ids.numel()].long()
            ids = torch.where(src >= 0, toks.long()[src.clamp(min=0)], ids.long())
        return table[ids.long()].clone()
    if out is None:
        out = torch.empty(ids.numel(), table.shape[1], dtype=table.dtype, device=ids.device)
    native().embed(ids, table, out, status_word(ids.device), *(feed if feed is not None else (None, None)))
    count_launches()
    return out


def rmsnorm(x, weight, eps, residual=None, out=None):
    """Reference numerics (layernorm.py:18-38).  With ``residual`` the sum
    x + residual is written back into ``residual`` (the new residual stream)."""
    if not x.is_cuda:
        xf = x.float()
        if residual is not None:
            xf = xf + residual.float()
            residual.copy_(xf.to(residual.dtype))
        var = xf.pow(2).mean(dim=-1, keepdim=True)
        y = (xf * torch.rsqrt(var + eps)).to(x.dtype) * weight
        return y if out is None else out.copy_(y)
    if out is None:
        out = torch.empty_like(x)
    native().rmsnorm(x, residual, weight, out, residual, eps)
    count_launches()
    return out


def moe_combine_add_rmsnorm(slots, topk, residual, weight, eps, out=None, zero=None, wait=None):
    """residual += sum_k slots[t, k] (fixed order); return rmsnorm(residual).
    ``zero``: an int32 buffer the kernel also clears (the layer's routing counters).
    ``wait`` = (done flags [W], epoch, status, wait_ns): expert parallelism, the kernel
    first waits (bounded) until every owner has released this layer's epoch."""
    T, H = residual.shape
    if not residual.is_cuda:
        if zero is not None:
            zero.zero_()
        moe = slots[:T * topk].view(T, topk, H).float().sum(dim=1).to(residual.dtype)
        return rmsnorm(moe, weight, eps, residual=residual, out=out)
    if out is None:
        out = torch.empty_like(residual)
    flags, epoch, status, wait_ns = wait if wait is not None else (None, None, None, None)
    native().moe_combine(slots, topk, residual, weight, out, eps, zero, flags, epoch, status, wait_ns)
    count_launches()
    return out


def rope_cos_sin(head_dim: int, max_pos: int, theta: float, device) -> torch.Tensor:
    """[max_pos, head_dim] fp32: cos | sin of the neox rotary (rotary_embedding.py:18-35)."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float) / head_dim))
    t = torch.arange(max_pos, dtype=torch.float)
    freqs = torch.outer(t, inv_freq)
    return torch.cat((freqs.cos(), freqs.sin()), dim=-1).to(device)


def qkv_norm_rope_kvstore(x, weight, scale, positions, slot_mapping, q_norm_w, k_norm_w, cos_sin, kv_layer, nq,
                          nkv, D, eps, qkv_out, q_out, tiled: bool = False):
    """QKV projection, then q/k RMSNorm + RoPE, q out and k/v into the paged pool.  When
    the planner splits the decode-size GEMM over K, the fp32 partials go straight into
    the norm kernel (summed there in split order: the bits of a separate reduction),
    one launch less per layer."""
    T, K = x.shape
    N = weight.shape[0]
    if x.is_cuda and scale is not None and weight.dim() == 2 and 0 < T < BF16_DENSE_ROWS:
        bn, splits = plan_dense(T, N // 128, K // 64, fp8=True)
        if splits > 1:
            part = torch.empty(splits * T, N, dtype=torch.float32, device=x.device)
            native().gemm(weight, scale, x, count_tensor(T, x.device), None, part, bn, EPI_F32, N // 128,
                          0, 0, None, None, status_word(x.device), _trace[0], splits, T * N, tiled, [])
            count_launches()
            return qknorm_rope_kvstore(qkv_out, positions, slot_mapping, q_norm_w, k_norm_w, cos_sin, kv_layer,
                                       nq, nkv, D, eps, q_out, part=part, splits=splits)
    qkv = linear(x, weight, scale, out=qkv_out, tiled=tiled)
    return qknorm_rope_kvstore(qkv, positions, slot_mapping, q_norm_w, k_norm_w, cos_sin, kv_layer, nq, nkv, D,
                               eps, q_out)


def qknorm_rope_kvstore(qkv, positions, slot_mapping, q_norm_w, k_norm_w, cos_sin, kv_layer, nq, nkv, D,
                        eps, q_out=None, part=None, splits: int = 1):
    """Normalise + rotate q/k, write k (rotated) and v into the paged pool
    (``kv_layer`` is a :class:`~b200moe.engine.kv_cache.KVLayer`).  ``part``: the
    QKV GEMM's fp32 split-K partials [splits * T, width] instead of ``qkv``."""
    T = qkv.shape[0]
    if q_out is None:
        q_out = torch.empty(T, nq, D, dtype=qkv.dtype, device=qkv.device)
    if not qkv.is_cuda:
        q = qkv[:, :nq * D].reshape(T, nq, D)
        k = qkv[:, nq * D:(nq + nkv) * D].reshape(T, nkv, D)
        v = qkv[:, (nq + nkv) * D:].reshape(T, nkv, D)

        def norm(x, w):
            xf = x.float()
            var = xf.pow(2).mean(dim=-1, keepdim=True)
            return (xf * torch.rsqrt(var + eps)).to(x.dtype) * w

        def rope(x):
            cs = cos_sin[positions.long()]
            c, s = cs.chunk(2, dim=-1)
            c, s = c.unsqueeze(1), s.unsqueeze(1)
            x1, x2 = x.float().chunk(2, dim=-1)
            return torch.cat((x1 * c - x2 * s, x2 * c + x1 * s), dim=-1).to(x.dtype)

        q_out.copy_(rope(norm(q, q_norm_w)))
        kv_layer.store(slot_mapping, rope(norm(k, k_norm_w)), v)
        return q_out
    native().qknorm_rope_kvstore(qkv, positions, slot_mapping, q_norm_w, k_norm_w, cos_sin, kv_layer.k,
                                 kv_layer.v, kv_layer.k_scale, kv_layer.v_scale, q_out, nq, nkv, D,
                                 kv_layer.block_size, kv_layer.block_stride, kv_layer.scale_block_stride, eps,
                                 part, splits, _chan_store(kv_layer))
    count_launches()
    return q_out


def router_topk(logits, num_experts, topk, renorm, ids, weights, counts=None):
    """Softmax over the first ``num_experts`` logit columns (rounded to bf16
    first, like the reference's bf16 gate output), top-k, renormalise, bf16
    weights; optionally add the per-expert counts into ``counts``."""
    if not logits.is_cuda:
        p = torch.softmax(logits[:, :num_experts].to(torch.bfloat16).float(), dim=-1)
        w, i = torch.topk(p, topk, dim=-1)
        if renorm:
            w = w / w.sum(dim=-1, keepdim=True)
        ids.copy_(i.to(ids.dtype))
        weights.copy_(w.to(torch.bfloat16).float())
        if counts is not None:
            counts.add_(torch.bincount(i.flatten(), minlength=counts.numel()).to(counts.dtype))
        return
    native().router_topk(logits, num_experts, topk, renorm, ids, weights, counts)
    count_launches()


_router_scratch: dict = {}


def router_scratch(device) -> tuple[torch.Tensor, torch.Tensor]:
    """Fixed-size per-device scratch of the split-K router (partial logits of up to
    2 x NUM_SMS tiles of 16 x 128, and zeroed per-tile counters).  Allocated on the
    first call -- an eager step, before any graph capture -- and never resized, so
    captured graphs keep valid addresses."""
    key = torch.device(device)
    s = _router_scratch.get(key)
    if s is None:
        s = (torch.empty(2 * NUM_SMS * 16 * 128, dtype=torch.float32, device=key),
             torch.zeros(2 * NUM_SMS, dtype=torch.int32, device=key))
        _router_scratch[key] = s
    return s


def router_fused(x, router_w, num_experts, topk, renorm, ids, weights, counts=None):
    """Router GEMM + softmax + top-k in one native launch (num_experts <= 128);
    same rounding points as ``linear`` + ``router_topk``.  Batches with too few
    16-token tiles to fill the SMs also split K across CTAs."""
    part, cnt = router_scratch(x.device)
    native().router_fused(x, router_w, num_experts, topk, renorm, ids, weights, counts, status_word(x.device),
                          part, cnt)
    count_launches()


def moe_permute(x, ids, counts, cursor, x_perm, slot_of_row, offsets_out=None):
    native().moe_permute(x, ids, counts, cursor, x_perm, slot_of_row, offsets_out)
    count_launches()


def _chan_read(kv_layer) -> list[int]:
    """Device pointers of the int8 channel mode's read side (attention kernels), or []."""
    c = kv_layer.chan
    if c is None:
        return []
    return [c.dscale.data_ptr(), c.out_idx.data_ptr(), c.n_out.data_ptr(), c.side_k.data_ptr(),
            c.side_v.data_ptr(), c.side_block_stride]


def _chan_store(kv_layer) -> list[int]:
    """Device pointers of the int8 channel mode's store side (KV-store kernel), or []."""
    c = kv_layer.chan
    if c is None:
        return []
    return [c.scale.data_ptr(), c.out_idx.data_ptr(), c.n_out.data_ptr(), c.side_k.data_ptr(), c.side_v.data_ptr(),
            c.side_block_stride, c.calib_amax.data_ptr() if c.calibrating else 0,
            c.calib_sum.data_ptr() if c.calibrating else 0]


def decode_attention(q, kv_layer, block_tables, seq_lens, scale, out, split_len, num_splits, workspace):
    """q [B, nq, D], one query per sequence; keys are the first seq_lens[b] slots."""
    if not q.is_cuda:
        return _attention_ref(q, kv_layer, block_tables, seq_lens,
                              torch.arange(q.shape[0] + 1, dtype=torch.int32), scale, out)
    part_o, part_m, part_l = workspace
    native().decode_attn(q, kv_layer.k, kv_layer.v, kv_layer.k_scale, kv_layer.v_scale, block_tables, seq_lens,
                         out, part_o, part_m, part_l, kv_layer.block_size, kv_layer.block_stride,
                         kv_layer.num_kv_heads, scale, num_splits, split_len, status_word(q.device),
                         _chan_read(kv_layer))
    count_launches(2 if num_splits > 1 else 1)
    return out


# int8 prefill: the referenced blocks are dequantised into a bf16 staging pool that
# the tcgen05 prefill kernel reads.  Above this many staging bytes per call the
# warp-MMA kernel that dequantises while staging runs instead.
INT8_STAGE_MAX_BYTES = int(os.environ.get("B200MOE_INT8_STAGE_MB", "2048")) << 20
_int8_stage: dict = {}


def _int8_stage_buffers(device, blocks: int, block_elems: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-device bf16 staging pool and identity block ids, grown on demand (prefill
    is never graph-captured, so growth cannot strand a captured address)."""
    key = torch.device(device)
    st = _int8_stage.get(key)
    if st is None or st[0].numel() < blocks * block_elems or st[1].numel() < blocks:
        st = (torch.empty(blocks * block_elems, dtype=torch.bfloat16, device=key),
              torch.arange(blocks, dtype=torch.int32, device=key))
        _int8_stage[key] = st
    return st


def _int8_prefill_staged(q, kv_layer, cu_seqlens_q, seq_lens, block_tables, max_q_len, scale, out) -> bool:
    """int8 pool, head_dim 128: stage the rows' blocks as bf16 (one launch) and run
    the tensor-core prefill on the stage (block b * max_blocks + j holds block j of
    row b).  Returns False where the tensor-core kernel does not take the shape."""
    D, nq = q.shape[2], q.shape[1]
    nkv, bs = kv_layer.num_kv_heads, kv_layer.block_size
    if (D != 128 or os.environ.get("B200MOE_PREFILL_TC") == "0" or os.environ.get("B200MOE_INT8_STAGE") == "0"
            or 128 % (nq // nkv) or not (bs % 128 == 0 or (128 % bs == 0 and bs % 8 == 0))):
        return False
    B, mb = block_tables.shape
    block_elems = 2 * nkv * bs * D
    if B * mb * block_elems * 2 > INT8_STAGE_MAX_BYTES:
        return False
    stage, ids = _int8_stage_buffers(q.device, B * mb, block_elems)
    native().kv_int8_stage(kv_layer.k, kv_layer.v, kv_layer.k_scale, kv_layer.v_scale, block_tables, seq_lens,
                           stage, bs, kv_layer.block_stride, nkv, _chan_read(kv_layer))
    st = stage[:B * mb * block_elems].view(B * mb, 2, nkv * bs * D)
    native().prefill_attn(q, st[:, 0], st[:, 1], None, None, cu_seqlens_q, seq_lens, ids[:B * mb].view(B, mb), out,
                          max_q_len, bs, block_elems, nkv, scale, status_word(q.device), [])
    count_launches(2)
    return True


def prefill_attention(q, kv_layer, cu_seqlens_q, seq_lens, block_tables, max_q_len, scale, out):
    if not q.is_cuda:
        return _attention_ref(q, kv_layer, block_tables, seq_lens, cu_seqlens_q, scale, out)
    if kv_layer.k.dtype == torch.int8 and _int8_prefill_staged(q, kv_layer, cu_seqlens_q, seq_lens, block_tables,
                                                               max_q_len, scale, out):
        return out
    native().prefill_attn(q, kv_layer.k, kv_layer.v, kv_layer.k_scale, kv_layer.v_scale, cu_seqlens_q, seq_lens,
                          block_tables, out, max_q_len, kv_layer.block_size, kv_layer.block_stride,
                          kv_layer.num_kv_heads, scale, status_word(q.device), _chan_read(kv_layer))
    count_launches()
    return out


def _attention_ref(q, kv_layer, block_tables, seq_lens, cu_seqlens_q, scale, out):
    """fp32 causal attention over the paged pool, one sequence at a time."""
    nq, D = q.shape[1], q.shape[2]
    nkv = kv_layer.num_kv_heads
    G = nq // nkv
    cu = cu_seqlens_q.tolist()
    lens = seq_lens.tolist()
    for b in range(len(lens)):
        q0, q1 = cu[b], cu[b + 1]
        qlen, L = q1 - q0, lens[b]
        if qlen == 0:
            continue
        k, v = kv_layer.gather(block_tables[b], L)  # [L, nkv, D]
        qf = q[q0:q1].float().view(qlen, nkv, G, D)
        s = torch.einsum("qhgd,khd->hgqk", qf, k.float()) * scale
        qpos = torch.arange(L - qlen, L, device=q.device).view(qlen, 1)
        kpos = torch.arange(L, device=q.device).view(1, L)
        s = s.masked_fill(kpos > qpos, float("-inf"))
        p = torch.softmax(s, dim=-1)
        o = torch.einsum("hgqk,khd->qhgd", p, v.float()).reshape(qlen, nq, D)
        out[q0:q1] = o.to(out.dtype)
    return out


# ---------------------------------------------------------------- sampler
def argmax(logits: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    if out is None:
        out = torch.empty(logits.shape[0], dtype=torch.int32, device=logits.device)
    if not logits.is_cuda:
        return out.copy_(logits.float().argmax(dim=-1).to(torch.int32))
    native().argmax(logits, out)
    count_launches()
    return out


def sample(logits, temperature, top_k, top_p, min_p, seeds, offsets, out=None, allow=None, allow_row=None,
           logprobs=None):
    """temperature / top-k / top-p / min-p / exponential-race sampling (greedy
    rows where temperature < 1e-3) in one kernel per row.

    ``allow`` [n_masks, ceil(V / 32)] int32 allowed-token bitmasks with ``allow_row``
    [B] (mask of each row, -1 = unconstrained): guided decoding.  ``logprobs`` =
    (k, top_v [B, k] f32, top_i [B, k] i32, chosen [B] f32) receives the
    log-probabilities of the distribution each row sampled from (greedy rows: the
    raw logits under the mask); top_i is -1 where fewer than k tokens survive."""
    if out is None:
        out = torch.empty(logits.shape[0], dtype=torch.int32, device=logits.device)
    if not logits.is_cuda:
        toks, lp = sample_reference(logits, temperature, top_k, top_p, min_p, seeds, offsets, allow, allow_row,
                                    logprobs[0] if logprobs else 0)
        if logprobs:
            k, tv, ti, ch = logprobs
            tv.copy_(lp[0])
            ti.copy_(lp[1])
            ch.copy_(lp[2])
        return out.copy_(toks)
    k, tv, ti, ch = logprobs if logprobs else (0, None, None, None)
    native().sample(logits, temperature, top_k, top_p, min_p, seeds, offsets, out, allow, allow_row, k, tv, ti, ch)
    count_launches()
    return out


def sample_keep_reference(x: torch.Tensor, top_k: int, top_p: float, min_p: float) -> torch.Tensor:
    """Tokens a sampled row may draw, from its scaled logits ``x`` (-inf = masked):
    the sorted-vocabulary definition of top-k, then top-p over the top-k survivors,
    then min-p; ties at a threshold are kept (the kernel's radix select keeps them)."""
    V = x.shape[0]
    keep = torch.isfinite(x)
    if 0 < top_k < V:
        kth = torch.topk(x, top_k).values[-1]
        keep &= x >= kth
    if top_p < 1.0:
        xs = torch.where(keep, x, torch.tensor(float("-inf")))
        p = torch.softmax(xs, dim=-1)
        sp, si = torch.sort(p, descending=True)
        cum = sp.cumsum(0)
        n_keep = int((cum - sp < top_p).sum())
        keep &= x >= xs[si[max(n_keep, 1) - 1]]
    if min_p > 0:
        keep &= x >= x.max() + math.log(min_p)
    return keep


def sample_reference(logits, temperature, top_k, top_p, min_p, seeds, offsets, allow=None, allow_row=None,
                     lp_k: int = 0):
    """CPU sampler with the same filters (sorted-vocabulary definition) and a torch
    generator per row in place of Philox.  Returns (tokens, (top_v, top_i, chosen))
    with the log-probabilities of each row's distribution (None when lp_k = 0)."""
    B, V = logits.shape
    out = torch.empty(B, dtype=torch.int32)
    tv = torch.full((B, max(lp_k, 1)), float("-inf"))
    ti = torch.full((B, max(lp_k, 1)), -1, dtype=torch.int32)
    ch = torch.empty(B)
    for r in range(B):
        row = logits[r].float().cpu()
        if allow is not None and int(allow_row[r]) >= 0:
            words = allow[int(allow_row[r])].cpu().to(torch.int64) & 0xFFFFFFFF
            bits = torch.arange(V)
            ok = ((words[bits // 32] >> (bits % 32)) & 1).bool()
            row = torch.where(ok, row, torch.tensor(float("-inf")))
        t = float(temperature[r])
        if t < 1e-3:
            x, keep = row, torch.isfinite(row)
            tok = int(row.argmax())
        else:
            x = row / t
            keep = sample_keep_reference(x, int(top_k[r]) if top_k is not None else -1,
                                         float(top_p[r]) if top_p is not None else 1.0,
                                         float(min_p[r]) if min_p is not None else 0.0)
            g = torch.Generator().manual_seed(int(seeds[r]) + int(offsets[r] if offsets is not None else 0))
            e = torch.empty(V).exponential_(1.0, generator=g)
            score = torch.where(keep, x - x.max() - e.log(), torch.tensor(float("-inf")))
            tok = int(score.argmax())
        out[r] = tok
        if lp_k:
            lp = torch.log_softmax(torch.where(keep, x, torch.tensor(float("-inf"))), dim=-1)
            ch[r] = lp[tok]
            n = min(lp_k, int(keep.sum()))
            v, i = lp.topk(n)
            tv[r, :n], ti[r, :n] = v, i.to(torch.int32)
    return out, ((tv[:, :lp_k], ti[:, :lp_k], ch) if lp_k else None)


def apply_penalties(logits, rows, ids, gen_counts, presence, frequency, repetition):
    if not logits.is_cuda:
        r, i = rows.long(), ids.long()
        vals = logits[r, i]
        rep = repetition[r]
        vals = torch.where(vals < 0, vals * rep, vals / rep)
        gc = gen_counts.float()
        vals = torch.where(gc > 0, vals - presence[r] - frequency[r] * gc, vals)
        logits[r, i] = vals
        return logits
    native().penalties(logits, rows, ids, gen_counts, presence, frequency, repetition)
    count_launches()
    return logits
