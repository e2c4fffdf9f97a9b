"""Multi-process rollout orchestration (reference: orchestrator/*)."""
from .orchestrator import Orchestrator
from .types import GroupConfig, GroupResult, RewardFn, RolloutTask, per_rollout

__all__ = ["Orchestrator", "GroupConfig", "GroupResult", "RewardFn", "RolloutTask", "per_rollout"]
