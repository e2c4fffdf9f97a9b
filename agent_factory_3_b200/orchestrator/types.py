"""Orchestrator data types (reference: orchestrator/types.py:9-84)."""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Callable, Optional, Union

from ..rollout.parallel.config import RolloutConfig, RolloutResult


@dataclass
class RolloutTask:
    config: RolloutConfig
    server_url: str
    group_id: str
    index_in_group: int


@dataclass
class GroupConfig:
    group_id: str
    rollout_configs: list[RolloutConfig]
    metadata: dict[str, Any] = field(default_factory=dict)
    server_affinity: bool = False     # whole group on one server (shared prefix cache)


@dataclass
class GroupResult:
    group_id: str
    results: list[RolloutResult]
    rewards: list[float]
    metadata: dict[str, Any] = field(default_factory=dict)
    # filled by SampleProcessor
    advantages: list[float] = field(default_factory=list)
    trainable_mask: list[bool] = field(default_factory=list)
    skip_reasons: list[Optional[str]] = field(default_factory=list)
    filter_reason: Optional[str] = None
    reward_baseline: float = 0.0


RewardFn = Callable[[list[RolloutResult], dict[str, Any]], list[float]]
RewardReturn = Union[float, tuple[float, dict[str, float]]]


def per_rollout(fn: Callable[[RolloutResult, dict[str, Any]], RewardReturn]) -> RewardFn:
    """Lift a per-rollout reward to a group reward; a (reward, components) return also stores
    the named components on the result."""

    def wrapped(results: list[RolloutResult], metadata: dict[str, Any]) -> list[float]:
        out = []
        for r in results:
            v = fn(r, metadata)
            if isinstance(v, tuple):
                v, comps = v
                r.reward_components = comps
            out.append(float(v))
        return out

    return wrapped
