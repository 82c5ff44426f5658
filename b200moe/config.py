"""Engine configuration.

Field names and defaults follow the reference's ``Config`` dataclass
(nanovllm/config.py:8-55) so ``LLM(model, **kwargs)`` call sites carry over.
Differences, all deliberate:

* ``kvcache_block_size`` may be any multiple of 16 up to 1024 (the reference
  asserts a multiple of 256, config.py:59); the paged kernels here take the
  block size as a runtime argument.
* the MoE always runs expert-parallel over every rank; the attention layout is
  chosen by ``attention_parallel`` ("dp": each rank owns whole sequences and
  their KV, "tp": heads are split across ranks).
* ``hf_config`` is a :class:`ModelArgs` parsed straight from ``config.json``
  (no network, no transformers version coupling), or a named preset.
* ``device`` selects the execution device: ``"cuda"`` runs the native sm_100a
  kernels, ``"cpu"`` runs the fp32 torch reference path (the numerics oracle).
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass, field, fields
from typing import Any

MOE_BACKENDS = ("fused", "nccl_a2a", "loop")
# reference backend names, accepted and mapped onto the native fused path
MOE_BACKEND_ALIASES = {"grouped_mm": "fused", "fused_grouped_mm": "fused", "bmm_dense": "fused",
                       "vllm_fused": "fused"}
SCHED_POLICIES = ("fcfs", "stall_free", "stall_free_lpm")


@dataclass
class ModelArgs:
    """Architecture of a Qwen3-MoE (or dense Qwen3) checkpoint."""

    model_type: str = "qwen3_moe"
    vocab_size: int = 151936
    hidden_size: int = 2048
    num_hidden_layers: int = 48
    num_attention_heads: int = 32
    num_key_value_heads: int = 4
    head_dim: int = 128
    intermediate_size: int = 6144
    moe_intermediate_size: int = 768
    num_experts: int = 128
    num_experts_per_tok: int = 8
    norm_topk_prob: bool = True
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1_000_000.0
    max_position_embeddings: int = 40960
    tie_word_embeddings: bool = False
    torch_dtype: str = "bfloat16"
    eos_token_id: int | None = 151645
    bos_token_id: int | None = None
    # fp8 block quantisation of the checkpoint (None = plain float weights)
    quant_block: tuple[int, int] | None = (128, 128)
    mlp_only_layers: tuple[int, ...] = ()
    decoder_sparse_step: int = 1
    extra: dict[str, Any] = field(default_factory=dict)

    @property
    def dtype(self):
        import torch
        return getattr(torch, self.torch_dtype) if isinstance(self.torch_dtype, str) else self.torch_dtype

    @property
    def is_moe(self) -> bool:
        return self.model_type == "qwen3_moe" and self.num_experts > 0

    def is_moe_layer(self, layer_id: int) -> bool:
        if not self.is_moe or layer_id in self.mlp_only_layers:
            return False
        return (layer_id + 1) % max(1, self.decoder_sparse_step) == 0

    @classmethod
    def from_dict(cls, d: dict) -> "ModelArgs":
        known = {f.name for f in fields(cls)}
        kw = {k: v for k, v in d.items() if k in known and k not in ("extra", "quant_block", "mlp_only_layers")}
        if "num_experts" not in d and "num_local_experts" in d:
            kw["num_experts"] = d["num_local_experts"]
        if "rope_theta" not in d:
            rp = d.get("rope_parameters") or d.get("rope_scaling") or {}
            if isinstance(rp, dict) and "rope_theta" in rp:
                kw["rope_theta"] = rp["rope_theta"]
        if d.get("head_dim") is None:
            kw["head_dim"] = d["hidden_size"] // d["num_attention_heads"]
        if "dtype" in d and "torch_dtype" not in d and isinstance(d["dtype"], str):
            kw["torch_dtype"] = d["dtype"]
        eos = d.get("eos_token_id")
        if isinstance(eos, list):
            kw["eos_token_id"] = eos[0] if eos else None
        if d.get("model_type") == "qwen3":
            kw["num_experts"] = 0
        qc = d.get("quantization_config") or {}
        qblock = None
        if qc.get("quant_method") == "fp8":
            qblock = tuple(qc.get("weight_block_size") or (128, 128))
        args = cls(**kw, quant_block=qblock, mlp_only_layers=tuple(d.get("mlp_only_layers") or ()))
        args.extra = {k: v for k, v in d.items() if k not in known}
        return args

    def to_dict(self) -> dict:
        d = {f.name: getattr(self, f.name) for f in fields(self) if f.name not in ("extra", "quant_block")}
        d["mlp_only_layers"] = list(self.mlp_only_layers)
        d["num_local_experts"] = self.num_experts
        d["rope_scaling"] = None
        d["architectures"] = ["Qwen3MoeForCausalLM" if self.is_moe else "Qwen3ForCausalLM"]
        d["attention_bias"] = False
        d["hidden_act"] = "silu"
        if self.quant_block is not None:
            d["quantization_config"] = {
                "quant_method": "fp8", "fmt": "e4m3", "activation_scheme": "dynamic",
                "weight_block_size": list(self.quant_block),
            }
        return d

    @classmethod
    def from_pretrained(cls, path: str) -> "ModelArgs":
        with open(os.path.join(path, "config.json")) as f:
            return cls.from_dict(json.load(f))


# Named architectures used by tests and benchmarks (random-init; no download).
PRESETS: dict[str, dict] = {
    # BASELINE tiny config: 2 layers, hidden 256, 4q/2kv heads of 64, 8 experts top-2, fp32.
    "tiny-moe": dict(vocab_size=1024, hidden_size=256, num_hidden_layers=2, num_attention_heads=4,
                     num_key_value_heads=2, head_dim=64, moe_intermediate_size=128, num_experts=8,
                     num_experts_per_tok=2, intermediate_size=512, max_position_embeddings=4096,
                     rope_theta=1_000_000.0, torch_dtype="float32", eos_token_id=1023, quant_block=None),
    # Same shapes, fp8 block-quantised bf16 model (GPU tests of the native path).
    "tiny-moe-fp8": dict(vocab_size=1024, hidden_size=256, num_hidden_layers=2, num_attention_heads=4,
                         num_key_value_heads=2, head_dim=64, moe_intermediate_size=128, num_experts=8,
                         num_experts_per_tok=2, intermediate_size=512, max_position_embeddings=4096,
                         rope_theta=1_000_000.0, torch_dtype="bfloat16", eos_token_id=1023),
    # 30B-A3B geometry (real head / expert shapes) with 4 layers: fast GPU tests.
    "qwen3-30b-a3b-4l": dict(num_hidden_layers=4),
    "qwen3-30b-a3b": dict(),
    "qwen3-235b-a22b": dict(hidden_size=4096, num_hidden_layers=94, num_attention_heads=64,
                            num_key_value_heads=4, moe_intermediate_size=1536, intermediate_size=12288),
    # 235B-A22B geometry (hidden 4096, GQA group 16, experts 4096 x 1536) with 2 layers: GPU tests.
    "qwen3-235b-a22b-2l": dict(hidden_size=4096, num_hidden_layers=2, num_attention_heads=64,
                               num_key_value_heads=4, moe_intermediate_size=1536, intermediate_size=12288),
}


def preset_args(name: str) -> ModelArgs:
    spec = dict(PRESETS[name])
    qb = spec.pop("quant_block", (128, 128))
    args = ModelArgs(**spec)
    args.quant_block = qb
    return args


@dataclass
class Config:
    model: str
    max_num_batched_tokens: int = 16384
    max_num_seqs: int = 512
    max_model_len: int = 4096
    gpu_memory_utilization: float = 0.9
    tensor_parallel_size: int = 1
    enforce_eager: bool = False
    hf_config: ModelArgs | None = None
    eos: int = -1
    kvcache_block_size: int = 256
    num_kvcache_blocks: int = -1
    distributed_init_method: str = ""
    shm_name: str = ""
    expert_parallel_size: int = 0
    moe_backend: str = "fused"
    decode_moe_backend: str | None = None
    attention_backend: str = "paged"
    kv_cache_dtype: str = "bf16"
    # int8 KV quantisation: "token" (per token-head absmax scales) or "channel" (the
    # reference's calibrated per-channel scales + exact bf16 outlier dims)
    kv_int8_mode: str = "token"
    expert_placement: str = "linear"
    expert_map_path: str | None = None
    scheduler_policy: str = "fcfs"
    prefill_chunk_size: int = 256
    scheduler_starvation_steps: int = 32
    scheduler_overlap: bool = False
    kv_offload_enabled: bool = False
    kv_offload_host_blocks: int = 256
    metrics_path: str | None = None
    enable_profiling: bool = False
    # --- B200-native additions ---
    device: str = "cuda"
    attention_parallel: str = "dp"
    # random-init instead of loading weights ("" = load from `model`)
    random_init: str = ""
    seed: int = 0
    cuda_graph_max_bs: int = 512
    # bound on a worker rank's reply and on every collective (the process-group
    # timeout, which also bounds the ranks' start-up rendezvous: keep it above a
    # cold start's import time)
    rank_timeout_s: float = 120.0

    def __post_init__(self):
        if self.hf_config is None:
            if self.model in PRESETS and not os.path.isdir(self.model):
                self.hf_config = preset_args(self.model)
                if not self.random_init:
                    self.random_init = "seeded"
            else:
                if not os.path.isdir(self.model):
                    raise ValueError(f"model path {self.model!r} is not a directory or a known preset")
                self.hf_config = ModelArgs.from_pretrained(self.model)
        bs = self.kvcache_block_size
        if bs % 16 or not 16 <= bs <= 1024:
            raise ValueError("kvcache_block_size must be a multiple of 16 in [16, 1024]")
        if not 1 <= self.tensor_parallel_size <= 8:
            raise ValueError("tensor_parallel_size must be in [1, 8]")
        if self.expert_parallel_size == 0:
            self.expert_parallel_size = self.tensor_parallel_size
        if self.expert_parallel_size != self.tensor_parallel_size:
            raise ValueError("expert_parallel_size must equal the number of ranks (tensor_parallel_size)")
        a = self.hf_config
        if a.is_moe and a.num_experts % self.expert_parallel_size:
            raise ValueError("num_experts must be divisible by expert_parallel_size")
        self.moe_backend = MOE_BACKEND_ALIASES.get(self.moe_backend, self.moe_backend)
        if self.decode_moe_backend is not None:
            self.decode_moe_backend = MOE_BACKEND_ALIASES.get(self.decode_moe_backend, self.decode_moe_backend)
        if self.moe_backend not in MOE_BACKENDS:
            raise ValueError(f"moe_backend must be one of {MOE_BACKENDS}")
        if self.decode_moe_backend not in (None, *MOE_BACKENDS):
            raise ValueError(f"decode_moe_backend must be None or one of {MOE_BACKENDS}")
        if self.attention_backend == "triton_paged":
            self.attention_backend = "paged"
        if self.attention_backend not in ("paged", "sdpa"):
            raise ValueError("attention_backend must be 'paged' (native) or 'sdpa'")
        if self.kv_cache_dtype not in ("bf16", "int8"):
            raise ValueError("kv_cache_dtype must be 'bf16' or 'int8'")
        if self.kv_int8_mode not in ("token", "channel"):
            raise ValueError("kv_int8_mode must be 'token' or 'channel'")
        if self.kv_offload_enabled:
            if self.kv_cache_dtype != "bf16":
                raise ValueError("KV offload requires the bf16 KV cache")
            if self.kv_offload_host_blocks < 0:
                raise ValueError("kv_offload_host_blocks must be >= 0")
        if self.expert_placement not in ("linear", "round_robin", "profiled"):
            raise ValueError("expert_placement must be linear, round_robin or profiled")
        if self.expert_placement == "profiled" and not (self.expert_map_path and os.path.isfile(self.expert_map_path)):
            raise ValueError("profiled placement needs an existing expert_map_path")
        if self.scheduler_policy not in SCHED_POLICIES:
            raise ValueError(f"scheduler_policy must be one of {SCHED_POLICIES}")
        if self.prefill_chunk_size <= 0 or self.scheduler_starvation_steps <= 0:
            raise ValueError("prefill_chunk_size and scheduler_starvation_steps must be positive")
        if self.max_num_seqs > self.max_num_batched_tokens:
            raise ValueError("max_num_seqs must not exceed max_num_batched_tokens")
        if self.attention_parallel not in ("dp", "tp"):
            raise ValueError("attention_parallel must be 'dp' or 'tp'")
        if self.attention_parallel == "tp" and self.tensor_parallel_size > 1:
            heads, kvh, n = a.num_attention_heads, a.num_key_value_heads, self.tensor_parallel_size
            if heads % n or (kvh % n and n % kvh):
                raise ValueError("tp attention needs heads % tp == 0 and kv heads dividing or divisible by tp")
        if self.device not in ("cuda", "cpu"):
            raise ValueError("device must be 'cuda' or 'cpu'")
        self.max_model_len = min(self.max_model_len, a.max_position_embeddings)

    @property
    def world_size(self) -> int:
        return self.tensor_parallel_size

    @property
    def dp_size(self) -> int:
        return self.world_size if self.attention_parallel == "dp" else 1


def config_field_names() -> set[str]:
    return {f.name for f in fields(Config)}
