"""Per-rollout statistics: routing range check, generated tokens, number of rounds."""
from __future__ import annotations

import numpy as np

from ..types import ReactResult, StepType
from .config import RolloutResult


def validate_routing_indices(r: ReactResult, num_experts: int = 128) -> bool:
    if r.routing_indices is None:
        return True
    for ri in r.routing_indices:
        if ri is None:
            continue
        a = np.asarray(ri)
        if a.size and (a.min() < 0 or a.max() >= num_experts):
            return False
    return True


def compute_stats(result: RolloutResult, num_experts: int = 128) -> RolloutResult:
    if not result.success or result.result is None:
        return result
    rr = result.result
    return result.model_copy(update={
        "routing_valid": validate_routing_indices(rr, num_experts),
        "completion_tokens_count": rr.num_generated_tokens,
        "num_rounds": sum(1 for s in rr.steps if s.type == StepType.ASSISTANT)})


def compute_stats_batch(results: list[RolloutResult], num_experts: int = 128) -> list[RolloutResult]:
    return [compute_stats(r, num_experts) for r in results]
