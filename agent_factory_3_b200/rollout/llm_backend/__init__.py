"""LLM generation backends (reference: rollout/llm_backend/*)."""
from .protocol import LLMBackend
from .sglang_backend import SGLangBackend
from .types import GenerationResult

__all__ = ["LLMBackend", "SGLangBackend", "GenerationResult"]
