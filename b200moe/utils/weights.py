"""Weights: HF safetensors loader, random initialisation and checkpoint writer.

Checkpoint format (the one the reference loads, nanovllm/utils/loader.py:64-143):
HF Qwen3-MoE tensor names; with ``quantization_config.quant_method == "fp8"``
the linear and expert weights are e4m3 with an fp32 ``<name>_scale_inv`` per
128x128 block.  Unlike the reference, which dequantises every weight to bf16 on
the CPU at load, the e4m3 bytes and their scales stay as they are on the
device (half the HBM; the GEMM dequantises per tile in shared memory).

Packing (checkpoint name -> parameter):
  self_attn.{q,k,v}_proj          -> layers[l].qkv_weight rows [q | k | v]
  self_attn.o_proj                -> layers[l].o_weight
  mlp.experts.{e}.{gate,up}_proj  -> layers[l].w13[local(e)] rows [gate | up]
  mlp.experts.{e}.down_proj       -> layers[l].w2[local(e)]
  mlp.gate                        -> layers[l].router (rows padded to 128)
  mlp.{gate,up,down}_proj (dense) -> layers[l].w13[0] / w2[0]
Experts not owned by this rank are skipped; every parameter must be written
(coverage check, as the reference's _assert_full_coverage, loader.py:146-163).
"""
from __future__ import annotations

import contextlib
import json
import os
from glob import glob

import torch

from b200moe.config import ModelArgs

FP8_MAX = 448.0


# ------------------------------------------------------------ quantisation
def quantize_block_fp8(w: torch.Tensor, block: int = 128) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-128x128-block absmax e4m3 quantisation: w ~= q * scale_inv."""
    *lead, N, K = w.shape
    wb = w.float().reshape(*lead, N // block, block, K // block, block)
    amax = wb.abs().amax(dim=(-3, -1), keepdim=True).clamp_min(1e-12)
    scale = amax / FP8_MAX
    q = (wb / scale).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)
    return q.reshape(*lead, N, K), scale.reshape(*lead, N // block, K // block).contiguous()


# ------------------------------------------------------------- random init
@contextlib.contextmanager
def natural_layout(model):
    """Give the body the row-major weight layout that loaders and exporters
    index; tile-major GEMM weights (model.tile_weights_) are restored after."""
    tiled = getattr(model, "weights_tiled", False)
    if tiled:
        model.untile_weights_()
    try:
        yield
    finally:
        if tiled:
            model.tile_weights_()


@torch.no_grad()
def random_init_(model, seed: int = 0, std: float = 0.02):
    with natural_layout(model):
        _random_init(model, seed, std)


def _random_init(model, seed: int = 0, std: float = 0.02):
    """Seeded normal(0, std) init of every weight directly on the model's
    device (norm weights stay 1).  Quantised weights are drawn in fp32 and
    block-quantised, so the bytes look like a real fp8 checkpoint.  Expert
    tensors are drawn per global expert id, so every expert-parallel rank gets
    the same values for an expert whatever the placement."""
    dev = model.device
    args: ModelArgs = model.args

    def gen(shape, key):
        g = torch.Generator(device=dev)
        g.manual_seed((seed * 1_000_003 + key) & 0x7FFFFFFFFFFF)
        return torch.randn(*shape, generator=g, device=dev, dtype=torch.float32) * std

    def fill2d(param, scale_param, key):
        if scale_param is None:
            param.copy_(gen(param.shape, key).to(param.dtype))
        else:
            q, s = quantize_block_fp8(gen(param.shape, key))
            param.copy_(q)
            scale_param.copy_(s)

    def fill_sliced(param, scale_param, key, full_shape, rows=None, cols=None):
        """Draw the full weight (so every tensor-parallel rank holds a slice of
        the same tensor), quantise it blockwise, keep this rank's rows / cols."""
        full = gen(full_shape, key)
        if scale_param is not None:
            for lo, hi in (rows or []) + ([cols] if cols else []):
                if lo % 128 or hi % 128:
                    raise ValueError("tensor-parallel slices of fp8 weights must be 128-aligned")
            q, sc = quantize_block_fp8(full)
        else:
            q, sc = full.to(param.dtype), None
        if rows is not None:
            param.copy_(torch.cat([q[a:b] for a, b in rows]))
            if sc is not None:
                scale_param.copy_(torch.cat([sc[a // 128:b // 128] for a, b in rows]))
        else:
            a, b = cols
            param.copy_(q[:, a:b])
            if sc is not None:
                scale_param.copy_(sc[:, a // 128:b // 128])

    model.embed_tokens.copy_(gen(model.embed_tokens.shape, 1).to(model.embed_tokens.dtype))
    if model.lm_head is not model.embed_tokens:
        model.lm_head.copy_(gen(model.lm_head.shape, 2).to(model.lm_head.dtype))
    for l, layer in enumerate(model.layers):
        base = 100 + 16 * l
        if getattr(model, "attn_tp", 1) > 1:
            D = args.head_dim
            nqkv = (args.num_attention_heads + 2 * args.num_key_value_heads) * D
            fill_sliced(layer.qkv_weight, layer.qkv_scale, base + 1, (nqkv, args.hidden_size),
                        rows=model.qkv_row_ranges())
            fill_sliced(layer.o_weight, layer.o_scale, base + 2, (args.hidden_size, args.num_attention_heads * D),
                        cols=model.o_col_range())
        else:
            fill2d(layer.qkv_weight, layer.qkv_scale, base + 1)
            fill2d(layer.o_weight, layer.o_scale, base + 2)
        if layer.is_moe:
            E = args.num_experts
            layer.router.zero_()
            layer.router[:E].copy_(gen((E, args.hidden_size), base + 3).to(layer.router.dtype))
            experts = list(enumerate(model.expert_ids))
        else:
            experts = [(0, -1)]
        for le, ge in experts:
            k13 = (base + 4) * 4096 + ge + 1
            k2 = (base + 5) * 4096 + ge + 1
            fill2d(layer.w13[le], None if layer.s13 is None else layer.s13[le], k13)
            fill2d(layer.w2[le], None if layer.s2 is None else layer.s2[le], k2)


# ----------------------------------------------------------------- export
@torch.no_grad()
def export_state(model) -> dict[str, torch.Tensor]:
    """HF-named tensors of a model that holds every expert."""
    with natural_layout(model):
        return _export_state(model)


def _export_state(model) -> dict[str, torch.Tensor]:
    args: ModelArgs = model.args
    if args.is_moe and model.num_local_experts != args.num_experts:
        raise ValueError("export needs a model holding every expert")
    D = args.head_dim
    nq, nkv = args.num_attention_heads, args.num_key_value_heads
    out: dict[str, torch.Tensor] = {
        "model.embed_tokens.weight": model.embed_tokens,
        "model.norm.weight": model.norm,
    }
    if not args.tie_word_embeddings:
        out["lm_head.weight"] = model.lm_head

    def put(name, w, s, rows=None):
        out[name + ".weight"] = w if rows is None else w[rows[0]:rows[1]]
        if s is not None:
            out[name + ".weight_scale_inv"] = s if rows is None else s[rows[0] // 128:rows[1] // 128]

    for l, layer in enumerate(model.layers):
        p = f"model.layers.{l}."
        out[p + "input_layernorm.weight"] = layer.input_layernorm
        out[p + "post_attention_layernorm.weight"] = layer.post_attention_layernorm
        out[p + "self_attn.q_norm.weight"] = layer.q_norm
        out[p + "self_attn.k_norm.weight"] = layer.k_norm
        bounds = [0, nq * D, (nq + nkv) * D, (nq + 2 * nkv) * D]
        for i, n in enumerate(("q_proj", "k_proj", "v_proj")):
            put(p + "self_attn." + n, layer.qkv_weight, layer.qkv_scale, (bounds[i], bounds[i + 1]))
        put(p + "self_attn.o_proj", layer.o_weight, layer.o_scale)
        I = layer.w2.shape[-1]

        def mlp(prefix, e):
            s13 = None if layer.s13 is None else layer.s13[e]
            put(prefix + "gate_proj", layer.w13[e], s13, (0, I))
            put(prefix + "up_proj", layer.w13[e], s13, (I, 2 * I))
            put(prefix + "down_proj", layer.w2[e], None if layer.s2 is None else layer.s2[e])

        if layer.is_moe:
            out[p + "mlp.gate.weight"] = layer.router[:args.num_experts]
            for e in range(args.num_experts):
                mlp(f"{p}mlp.experts.{e}.", e)
        else:
            mlp(p + "mlp.", 0)
    return {k: v.detach().contiguous().cpu() for k, v in out.items()}


def save_checkpoint(model, path: str, max_shard_bytes: int = 4 << 30):
    """Write config.json + model-*.safetensors in the HF fp8 layout."""
    from safetensors.torch import save_file
    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(model.args.to_dict(), f, indent=1)
    state = export_state(model)
    shards, cur, size = [], {}, 0
    for k in sorted(state):
        t = state[k]
        nbytes = t.numel() * t.element_size()
        if cur and size + nbytes > max_shard_bytes:
            shards.append(cur)
            cur, size = {}, 0
        cur[k] = t
        size += nbytes
    if cur:
        shards.append(cur)
    index = {}
    for i, shard in enumerate(shards):
        name = f"model-{i + 1:05d}-of-{len(shards):05d}.safetensors"
        save_file(shard, os.path.join(path, name), metadata={"format": "pt"})
        for k in shard:
            index[k] = name
    with open(os.path.join(path, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {}, "weight_map": index}, f)


# ------------------------------------------------------------------- load
@torch.no_grad()
def load_checkpoint(model, path: str):
    """Load an HF checkpoint into ``model`` (this rank's experts only)."""
    with natural_layout(model):
        _load_checkpoint(model, path)


def _load_checkpoint(model, path: str):
    from safetensors import safe_open
    args: ModelArgs = model.args
    D = args.head_dim
    nq, nkv = args.num_attention_heads, args.num_key_value_heads
    keymap: dict[str, str] = {}
    for file in sorted(glob(os.path.join(path, "*.safetensors"))):
        with safe_open(file, "pt", "cpu") as f:
            for k in f.keys():
                keymap[k] = file
    if not keymap:
        raise FileNotFoundError(f"no *.safetensors under {path}")
    handles: dict[str, object] = {}

    def get(name):
        if name not in keymap:
            raise KeyError(f"checkpoint is missing {name}")
        file = keymap[name]
        h = handles.get(file)
        if h is None:
            h = safe_open(file, "pt", "cpu")
            handles[file] = h
        t = h.get_tensor(name)
        if t.dtype == torch.uint8:
            t = t.view(torch.float8_e4m3fn)
        return t

    def copy_into(dst: torch.Tensor, src: torch.Tensor):
        if tuple(dst.shape) != tuple(src.shape):
            raise ValueError(f"shape mismatch {tuple(src.shape)} -> {tuple(dst.shape)}")
        if dst.dtype == torch.float8_e4m3fn and src.dtype != torch.float8_e4m3fn:
            raise ValueError("checkpoint weight is not fp8 but the model expects fp8")
        dst.copy_(src if dst.dtype == torch.float8_e4m3fn else src.to(dst.dtype))

    def weight_pair(name, dst_w, dst_s):
        copy_into(dst_w, get(name + ".weight"))
        if dst_s is not None:
            copy_into(dst_s, get(name + ".weight_scale_inv").float())

    copy_into(model.embed_tokens, get("model.embed_tokens.weight"))
    copy_into(model.norm, get("model.norm.weight"))
    if not args.tie_word_embeddings:
        copy_into(model.lm_head, get("lm_head.weight"))
    for l, layer in enumerate(model.layers):
        p = f"model.layers.{l}."
        for src, dst in (("input_layernorm", layer.input_layernorm),
                         ("post_attention_layernorm", layer.post_attention_layernorm),
                         ("self_attn.q_norm", layer.q_norm), ("self_attn.k_norm", layer.k_norm)):
            copy_into(dst, get(p + src + ".weight"))
        # this rank's rows of q / k / v (all of them unless attention is tensor-parallel)
        local = model.qkv_row_ranges() if hasattr(model, "qkv_row_ranges") else \
            [(0, nq * D), (nq * D, (nq + nkv) * D), ((nq + nkv) * D, (nq + 2 * nkv) * D)]
        starts = [0, nq * D, (nq + nkv) * D]
        r = 0
        for i, n in enumerate(("q_proj", "k_proj", "v_proj")):
            a0, a1 = local[i][0] - starts[i], local[i][1] - starts[i]  # rows within this projection
            rows = a1 - a0
            w_src = get(p + "self_attn." + n + ".weight")[a0:a1]
            copy_into(layer.qkv_weight[r:r + rows], w_src)
            if layer.qkv_scale is not None:
                if a0 % 128 or a1 % 128:
                    raise ValueError("tensor-parallel slices of fp8 weights must be 128-aligned")
                s_src = get(p + "self_attn." + n + ".weight_scale_inv").float()[a0 // 128:a1 // 128]
                copy_into(layer.qkv_scale[r // 128:(r + rows) // 128], s_src)
            r += rows
        c0, c1 = model.o_col_range() if hasattr(model, "o_col_range") else (0, nq * D)
        copy_into(layer.o_weight, get(p + "self_attn.o_proj.weight")[:, c0:c1])
        if layer.o_scale is not None:
            copy_into(layer.o_scale, get(p + "self_attn.o_proj.weight_scale_inv").float()[:, c0 // 128:c1 // 128])
        I = layer.w2.shape[-1]

        def mlp(prefix, le):
            s13 = None if layer.s13 is None else layer.s13[le]
            weight_pair(prefix + "gate_proj", layer.w13[le, :I], None if s13 is None else s13[:I // 128])
            weight_pair(prefix + "up_proj", layer.w13[le, I:], None if s13 is None else s13[I // 128:])
            weight_pair(prefix + "down_proj", layer.w2[le], None if layer.s2 is None else layer.s2[le])

        if layer.is_moe:
            layer.router.zero_()
            copy_into(layer.router[:args.num_experts], get(p + "mlp.gate.weight"))
            for le, ge in enumerate(model.expert_ids):
                mlp(f"{p}mlp.experts.{ge}.", le)
        else:
            mlp(p + "mlp.", 0)
