"""Unified generation result of all backends."""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Optional


@dataclass
class GenerationResult:
    token_ids: list[int]
    finish_reason: Optional[str]            # "stop" | "length" | "abort" | None
    logprobs: Optional[list[float]]
    top_logprobs: Optional[list[dict[int, float]]]
    routing_indices: Optional[Any]          # np.ndarray uint8 [N-1, L, K] over prompt+completion
    cached_tokens: Optional[int]
    usage: Optional[dict[str, Any]]
    entropy: Optional[list[float]] = None
    weight_version: Optional[str] = None
