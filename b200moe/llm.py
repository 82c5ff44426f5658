"""``LLM`` is the offline engine (reference: nanovllm/llm.py:4)."""
from b200moe.engine.llm_engine import LLMEngine


class LLM(LLMEngine):
    pass
