"""Reference arm of bench.py: the UNMODIFIED reference engine (installed into
baseline/_ref) on the same workload, through its own public API
(``nanovllm.LLM(...).generate``).

The reference loads weights from disk, so this script first writes a random-init
checkpoint of the named architecture in the reference's format (HF names,
e4m3 weights + fp32 ``weight_scale_inv`` per 128x128 block, bf16 norms /
embeddings / router) plus a minimal HF tokenizer.  Only torch, safetensors
and tokenizers are used for that; nothing from b200moe is imported here.

Limits of the reference decide what can run (its tensor-parallel attention
asserts ``num_kv_heads % tp == 0``: Qwen3-30B-A3B has 4 KV heads, so 8 GPUs
cannot run); those cases print an ``unavailable`` line.
"""
from __future__ import annotations

import json
import os
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")
COMPLETE = ".checkpoint_complete"

ARCH = {
    "qwen3-30b-a3b": dict(hidden_size=2048, num_hidden_layers=48, num_attention_heads=32, num_key_value_heads=4,
                          head_dim=128, moe_intermediate_size=768, num_experts=128, num_experts_per_tok=8,
                          intermediate_size=6144, vocab_size=151936),
    "qwen3-30b-a3b-4l": dict(hidden_size=2048, num_hidden_layers=4, num_attention_heads=32, num_key_value_heads=4,
                             head_dim=128, moe_intermediate_size=768, num_experts=128, num_experts_per_tok=8,
                             intermediate_size=6144, vocab_size=151936),
}


def write_checkpoint(path: str, arch: dict, seed: int = 0, device: str = "cuda"):
    """Random-init Qwen3-MoE FP8 checkpoint (HF layout) + tokenizer at ``path``."""
    import torch
    from safetensors.torch import save_file
    os.makedirs(path, exist_ok=True)
    a = arch
    cfg = {
        "architectures": ["Qwen3MoeForCausalLM"], "model_type": "qwen3_moe", "hidden_act": "silu",
        "hidden_size": a["hidden_size"], "num_hidden_layers": a["num_hidden_layers"],
        "num_attention_heads": a["num_attention_heads"], "num_key_value_heads": a["num_key_value_heads"],
        "head_dim": a["head_dim"], "intermediate_size": a["intermediate_size"],
        "moe_intermediate_size": a["moe_intermediate_size"], "num_experts": a["num_experts"],
        "num_experts_per_tok": a["num_experts_per_tok"], "norm_topk_prob": True, "vocab_size": a["vocab_size"],
        "max_position_embeddings": 40960, "rms_norm_eps": 1e-6, "rope_theta": 1000000.0, "rope_scaling": None,
        "attention_bias": False, "tie_word_embeddings": False, "torch_dtype": "bfloat16", "decoder_sparse_step": 1,
        "mlp_only_layers": [], "bos_token_id": 151643, "eos_token_id": 151645,
        "quantization_config": {"quant_method": "fp8", "fmt": "e4m3", "activation_scheme": "dynamic",
                                "weight_block_size": [128, 128]},
    }
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(cfg, f, indent=1)
    _write_tokenizer(path, a["vocab_size"])
    g = torch.Generator(device=device).manual_seed(seed)
    H, D = a["hidden_size"], a["head_dim"]
    nq, nkv, I, E = a["num_attention_heads"], a["num_key_value_heads"], a["moe_intermediate_size"], a["num_experts"]

    def rnd(*shape):
        return torch.randn(*shape, generator=g, device=device) * 0.02

    def fp8(w):
        """[..., n, k] fp32 -> (e4m3 [..., n, k], fp32 scale_inv [..., n/128, k/128]) on the host,
        one device->host copy for the whole stack."""
        *lead, n, k = w.shape
        b = w.reshape(*lead, n // 128, 128, k // 128, 128)
        amax = b.abs().amax(dim=(-3, -1), keepdim=True).clamp_min(1e-12)
        s = amax / 448.0
        q = (b / s).clamp(-448, 448).to(torch.float8_e4m3fn).reshape(*lead, n, k)
        return q.cpu(), s.reshape(*lead, n // 128, k // 128).float().cpu()

    def put(d, name, w):
        q, s = fp8(w)
        d[name + ".weight"] = q
        d[name + ".weight_scale_inv"] = s

    bf = lambda t: t.to(torch.bfloat16).cpu()
    save_file({"model.embed_tokens.weight": bf(rnd(a["vocab_size"], H)), "lm_head.weight": bf(rnd(a["vocab_size"], H)),
               "model.norm.weight": bf(torch.ones(H))}, os.path.join(path, "model-embed.safetensors"))
    for l in range(a["num_hidden_layers"]):
        p = f"model.layers.{l}."
        d = {p + "input_layernorm.weight": bf(torch.ones(H)), p + "post_attention_layernorm.weight": bf(torch.ones(H)),
             p + "self_attn.q_norm.weight": bf(torch.ones(D)), p + "self_attn.k_norm.weight": bf(torch.ones(D)),
             p + "mlp.gate.weight": bf(rnd(E, H))}
        put(d, p + "self_attn.q_proj", rnd(nq * D, H))
        put(d, p + "self_attn.k_proj", rnd(nkv * D, H))
        put(d, p + "self_attn.v_proj", rnd(nkv * D, H))
        put(d, p + "self_attn.o_proj", rnd(H, nq * D))
        # all experts of a projection are drawn and quantised as one stack; safetensors
        # refuses tensors that share storage, so each expert's slice is cloned on the host
        for proj, shape in (("gate_proj", (I, H)), ("up_proj", (I, H)), ("down_proj", (H, I))):
            q, s = fp8(rnd(E, *shape))
            for e in range(E):
                name = f"{p}mlp.experts.{e}.{proj}"
                d[name + ".weight"] = q[e].clone()
                d[name + ".weight_scale_inv"] = s[e].clone()
        save_file(d, os.path.join(path, f"model-layer{l:03d}.safetensors"))
    with open(os.path.join(path, COMPLETE), "w") as f:  # written last: a partial checkpoint is rewritten
        f.write("ok\n")


def _write_tokenizer(path: str, vocab_size: int):
    from tokenizers import Tokenizer, models, pre_tokenizers
    vocab = {f"<{i}>": i for i in range(vocab_size)}
    tok = Tokenizer(models.WordLevel(vocab=vocab, unk_token="<0>"))
    tok.pre_tokenizer = pre_tokenizers.WhitespaceSplit()
    tok.save(os.path.join(path, "tokenizer.json"))
    with open(os.path.join(path, "tokenizer_config.json"), "w") as f:
        json.dump({"tokenizer_class": "PreTrainedTokenizerFast", "eos_token": "<151645>", "bos_token": "<151643>",
                   "pad_token": "<151643>", "unk_token": "<0>", "model_max_length": 40960}, f)


CKPT_BYTES = {"qwen3-30b-a3b": 33 << 30, "qwen3-30b-a3b-4l": 4 << 30}


def checkpoint_dir(model: str) -> str:
    """Where the random checkpoint goes: ``B200MOE_REF_CKPT`` if set, else the first of the
    system temp dir and the repository's ``_refckpt`` that has room for it (~31 GiB for
    the 30B model; a finished checkpoint is reused)."""
    import shutil
    import tempfile
    if os.environ.get("B200MOE_REF_CKPT"):
        return os.environ["B200MOE_REF_CKPT"]
    need = CKPT_BYTES.get(model, 40 << 30)
    for base in (tempfile.gettempdir(), os.path.join(ROOT, "_refckpt")):
        path = os.path.join(base, f"ref_ckpt_{model}")
        if os.path.exists(os.path.join(path, COMPLETE)):
            return path
        os.makedirs(base, exist_ok=True)
        if shutil.disk_usage(base).free >= need:
            return path
    return os.path.join(tempfile.gettempdir(), f"ref_ckpt_{model}")


class _Clocks:
    """``nvidia-smi`` SM clock and throttle-reason samples every 200 ms while the timed passes run."""

    FIELDS = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, n_gpus: int):
        import subprocess
        import tempfile
        self.log = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", ",".join(str(i) for i in range(n_gpus)), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.log, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"samples": 0}
        self.proc.terminate()
        self.proc.wait(timeout=10)
        self.log.seek(0)
        rows = [[c.strip() for c in line.split(",")] for line in self.log if line.count(",") == 5]
        os.unlink(self.log.name)
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        mhz = sorted(float(r[0]) for r in rows if r[0].replace(".", "").isdigit())
        return {"sm_mhz": mhz[len(mhz) // 2] if mhz else None,
                "sm_max_mhz": float(rows[0][1]) if rows and rows[0][1].replace(".", "").isdigit() else None,
                "reasons": [n for i, n in enumerate(names) if any(r[2 + i] == "Active" for r in rows)],
                "samples": len(rows)}


def unavailable(why: str) -> int:
    print(json.dumps({"impl": "reference", "unavailable": why}), flush=True)
    return 0


def run(args, prompts_for, metric: str) -> int:
    """``prompts_for(i)``: the prompts of pass i (fresh for every pass, like the main arm)."""
    if args.gpus > 4:
        return unavailable("reference asserts num_kv_heads % tp == 0 (nanovllm/models/qwen3.py:34); "
                           "Qwen3-30B-A3B has 4 KV heads, so 8 GPUs cannot run")
    if args.model not in ARCH:
        return unavailable(f"no reference-format checkpoint writer for {args.model}")
    if not os.path.isdir(os.path.join(REF, "nanovllm")):
        return unavailable(f"reference not installed: no package at {os.path.join(REF, 'nanovllm')}")
    import torch
    ckpt = checkpoint_dir(args.model)
    t0 = time.perf_counter()
    if not os.path.exists(os.path.join(ckpt, COMPLETE)):
        write_checkpoint(ckpt, ARCH[args.model], seed=args.seed)
    write_s = time.perf_counter() - t0
    sys.path.insert(0, REF)
    # Under torchrun, the agent-store flag would make the reference engine's own
    # rank 0 a client of its tcp:// rendezvous (no server): the reference is
    # normally started with plain python, so drop what torchrun adds.
    for var in ("TORCHELASTIC_USE_AGENT_STORE", "TORCHELASTIC_RESTART_COUNT"):
        os.environ.pop(var, None)
    from nanovllm import LLM, SamplingParams  # the reference package
    eager = os.environ.get("B200MOE_REF_EAGER", "1") != "0"
    # the reference's decode-only MoE backend (its config.decode_moe_backend); its
    # documentation names bmm_dense as the one its decode graphs can capture
    decode_moe = os.environ.get("B200MOE_REF_DECODE_MOE") or None
    t0 = time.perf_counter()
    llm = LLM(ckpt, tensor_parallel_size=args.gpus, max_num_seqs=max(args.num_requests, 1),
              max_num_batched_tokens=args.max_num_batched_tokens,
              max_model_len=args.input_len + args.output_len + 16, kvcache_block_size=256,
              moe_backend="grouped_mm", decode_moe_backend=decode_moe, attention_backend="triton_paged",
              scheduler_policy=args.scheduler_policy,
              # eager by default: the reference's production setting (its deploy/serve.env.example
              # and scripts/p2_benchmark.py run enforce_eager); B200MOE_REF_EAGER=0 tries its
              # CUDA-graph decode instead
              enforce_eager=eager)
    init_s = time.perf_counter() - t0
    sp = SamplingParams(temperature=0.0, max_tokens=args.output_len, ignore_eos=True)
    warm_s = []
    for i in range(args.warmup):
        tw = time.perf_counter()
        llm.generate(prompts_for(i), sp, use_tqdm=False)
        warm_s.append(round(time.perf_counter() - tw, 2))
    timed = [prompts_for(args.warmup + i) for i in range(args.steps)]
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk = _Clocks(args.gpus)
    a.record()
    t0 = time.perf_counter()
    total = 0
    for prompts in timed:
        outs = llm.generate(prompts, sp, use_tqdm=False)
        total += sum(len(o["token_ids"]) for o in outs)
    b.record()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    clocks = clk.stop()
    dev_s = a.elapsed_time(b) / 1e3
    ttft = sorted(o["metrics"]["ttft_s"] for o in outs if o["metrics"].get("ttft_s") is not None)
    tpot = sorted(o["metrics"]["tpot_s"] for o in outs if o["metrics"].get("tpot_s") is not None)
    line = {"impl": "reference", "metric": metric, "value": round(total / dev_s, 1), "unit": "tok/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(dev_s * 1e3 / args.steps, 1), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16 (reference dequantises the fp8 checkpoint at load)",
            "data": "synthetic uniform-random token ids; random-init fp8 checkpoint written at run time",
            "config": {"model": args.model, "global_batch": args.num_requests, "seq_len": args.input_len,
                       "output_len": args.output_len, "parallelism": f"tp{args.gpus}/ep{args.gpus}",
                       "moe_backend": "grouped_mm", "decode_moe_backend": decode_moe,
                       "attention_backend": "triton_paged", "enforce_eager": eager,
                       "ckpt_dir": ckpt, "ckpt_write_s": round(write_s, 1), "init_s": round(init_s, 1),
                       "warmup_pass_s": warm_s,
                       "timing": "CUDA events on rank 0's stream around the K passes; rank 0 waits on every "
                                 "collective, so this is the slowest rank's time"},
            "e2e": {"value": round(total / wall, 1), "unit": "tok/s", "wall_s_per_pass": round(wall / args.steps, 2)},
            "clocks": clocks}
    if ttft:
        line["p50_ttft_s"] = round(ttft[len(ttft) // 2], 4)
    if tpot:
        line["p50_tpot_s"] = round(tpot[len(tpot) // 2], 5)
    print(json.dumps(line), flush=True)
    llm.exit()
    return 0
