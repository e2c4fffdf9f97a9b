"""Per-rollout execution (MCP setup, conversation, runner) and a stand-alone batch runner."""
from .config import RolloutConfig, RolloutResult

__all__ = ["RolloutConfig", "RolloutResult"]
