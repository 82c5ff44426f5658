"""b200moe: a Mixture-of-Experts inference engine for NVIDIA B200 (sm_100a).

Public API (same shape as the reference's ``nanovllm`` package):
``from b200moe import LLM, SamplingParams``.
"""
from b200moe.llm import LLM
from b200moe.sampling_params import SamplingParams

__version__ = "0.1.0"

__all__ = ["LLM", "SamplingParams", "__version__"]
