"""Import alias: scripts written against the reference's ``nanovllm`` package
(``from nanovllm import LLM, SamplingParams``) run unchanged on b200moe."""
from b200moe import LLM, SamplingParams, __version__  # noqa: F401
