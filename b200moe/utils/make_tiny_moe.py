"""Write the tiny deterministic Qwen3-MoE checkpoint the test suites load from disk.

    python -m b200moe.utils.make_tiny_moe --out /tmp/tiny_moe [--tokenizer-from DIR]

Architecture (the reference's tiny test model, scripts/make_tiny_moe.py:22-49):
hidden 64, 4 query / 2 KV heads of dim 16, 2 layers, 8 experts top-2,
expert intermediate 32, vocab 151936, fp32, N(0, 0.02) weights (norms = 1).
head_dim 16 and hidden 64 are below the native kernels' tile sizes, so this
checkpoint exercises the CPU (fp32 oracle) path and the loader; GPU tests use
the ``tiny-moe-fp8`` preset instead.

Every tensor is drawn from its own generator seeded by (seed, tensor name), so
a tensor's values do not depend on the order tensors are written.  The
tokenizer files are copied from ``--tokenizer-from`` when given; otherwise a
word-level tokenizer over ``<id>`` tokens is written (no network needed).
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import shutil

import torch

TOKENIZER_FILES = ("tokenizer.json", "tokenizer_config.json", "vocab.json", "merges.txt")


def tiny_config() -> dict:
    return {
        "architectures": ["Qwen3MoeForCausalLM"], "model_type": "qwen3_moe",
        "hidden_size": 64, "head_dim": 16, "num_attention_heads": 4, "num_key_value_heads": 2,
        "num_hidden_layers": 2, "num_experts": 8, "num_experts_per_tok": 2, "moe_intermediate_size": 32,
        "intermediate_size": 32, "norm_topk_prob": True, "decoder_sparse_step": 1, "mlp_only_layers": [],
        "vocab_size": 151936, "max_position_embeddings": 4096, "rope_theta": 1000000, "rms_norm_eps": 1e-6,
        "tie_word_embeddings": False, "attention_bias": False, "torch_dtype": "float32",
        "eos_token_id": 151645, "pad_token_id": 151643, "bos_token_id": 151643,
    }


def _normal(name: str, shape, seed: int, std: float) -> torch.Tensor:
    key = int.from_bytes(hashlib.sha256(f"{seed}:{name}".encode()).digest()[:8], "little") & ((1 << 63) - 1)
    return torch.randn(*shape, generator=torch.Generator().manual_seed(key)) * std


def tiny_state(cfg: dict, seed: int = 0, std: float = 0.02) -> dict[str, torch.Tensor]:
    H, D = cfg["hidden_size"], cfg["head_dim"]
    nq, nkv, E, I = cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["num_experts"], \
        cfg["moe_intermediate_size"]
    shapes = {"model.embed_tokens.weight": (cfg["vocab_size"], H), "lm_head.weight": (cfg["vocab_size"], H)}
    ones = {"model.norm.weight": H}
    for l in range(cfg["num_hidden_layers"]):
        p = f"model.layers.{l}."
        ones.update({p + "input_layernorm.weight": H, p + "post_attention_layernorm.weight": H,
                     p + "self_attn.q_norm.weight": D, p + "self_attn.k_norm.weight": D})
        shapes.update({p + "self_attn.q_proj.weight": (nq * D, H), p + "self_attn.k_proj.weight": (nkv * D, H),
                       p + "self_attn.v_proj.weight": (nkv * D, H), p + "self_attn.o_proj.weight": (H, nq * D),
                       p + "mlp.gate.weight": (E, H)})
        for e in range(E):
            q = f"{p}mlp.experts.{e}."
            shapes.update({q + "gate_proj.weight": (I, H), q + "up_proj.weight": (I, H),
                           q + "down_proj.weight": (H, I)})
    state = {n: _normal(n, s, seed, std) for n, s in shapes.items()}
    state.update({n: torch.ones(d) for n, d in ones.items()})
    return state


def write_tiny_moe(out: str, seed: int = 0, tokenizer_from: str | None = None) -> str:
    from safetensors.torch import save_file
    os.makedirs(out, exist_ok=True)
    cfg = tiny_config()
    with open(os.path.join(out, "config.json"), "w") as f:
        json.dump(cfg, f, indent=2)
    save_file(tiny_state(cfg, seed), os.path.join(out, "model.safetensors"))
    if tokenizer_from:
        for name in TOKENIZER_FILES:
            src = os.path.join(tokenizer_from, name)
            if os.path.isfile(src):
                shutil.copy(src, os.path.join(out, name))
        missing = [n for n in TOKENIZER_FILES[:2] if not os.path.isfile(os.path.join(out, n))]
        if missing:
            raise FileNotFoundError(f"tokenizer files missing from {tokenizer_from}: {missing}")
    else:
        write_wordlevel_tokenizer(out, cfg["vocab_size"], cfg["eos_token_id"], cfg["bos_token_id"])
    return out


def write_wordlevel_tokenizer(out: str, vocab_size: int, eos_id: int, bos_id: int):
    """A whitespace word-level tokenizer whose token i is the word ``<i>``."""
    from tokenizers import Tokenizer, models, pre_tokenizers
    tok = Tokenizer(models.WordLevel(vocab={f"<{i}>": i for i in range(vocab_size)}, unk_token="<0>"))
    tok.pre_tokenizer = pre_tokenizers.WhitespaceSplit()
    tok.save(os.path.join(out, "tokenizer.json"))
    with open(os.path.join(out, "tokenizer_config.json"), "w") as f:
        json.dump({"tokenizer_class": "PreTrainedTokenizerFast", "eos_token": f"<{eos_id}>",
                   "bos_token": f"<{bos_id}>", "pad_token": f"<{bos_id}>", "unk_token": "<0>",
                   "model_max_length": 40960}, f)


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--out", default="/tmp/tiny_moe")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--tokenizer-from", default=None)
    args = p.parse_args(argv)
    write_tiny_moe(args.out, args.seed, args.tokenizer_from)
    n = sum(t.numel() for t in tiny_state(tiny_config(), args.seed).values())
    print(f"[make-tiny-moe] wrote {args.out} ({n * 4 / 1e6:.1f} MB fp32)")


if __name__ == "__main__":
    main()
