"""Per-rollout configuration and result (reference: rollout/parallel/config.py:11-77)."""
from __future__ import annotations

from typing import Any, Optional

from pydantic import BaseModel, ConfigDict, Field

from ..config import ConversationConfig, LoopConfig, RecordConfig
from ..types import ReactResult


class RolloutConfig(BaseModel):
    rollout_id: str
    user_prompt: str
    conv_config: ConversationConfig = Field(default_factory=ConversationConfig)
    loop_config: LoopConfig = Field(default_factory=LoopConfig)
    record_config: Optional[RecordConfig] = None
    mcp_config: Optional[dict[str, Any]] = None       # {"mcpServers": {ns: {command,args,env}}}
    metadata: dict[str, Any] = Field(default_factory=dict)


class RolloutResult(BaseModel):
    model_config = ConfigDict(arbitrary_types_allowed=True)

    rollout_id: str
    result: Optional[ReactResult] = None
    start_time: float
    end_time: float
    elapsed_time: float
    server_url: str
    success: bool
    error: Optional[str] = None
    traceback: Optional[str] = None
    routing_valid: Optional[bool] = None
    completion_tokens_count: Optional[int] = None
    num_rounds: Optional[int] = None
    weighted_reward: Optional[float] = None
    reward_components: Optional[dict[str, float]] = None

    @property
    def is_task_success(self) -> bool:
        return self.success and self.result is not None and self.result.is_success

    @property
    def end_reason(self) -> Optional[str]:
        return self.result.end_reason.value if self.result is not None else None

    @property
    def num_generated_tokens(self) -> int:
        return self.result.num_generated_tokens if self.result is not None else 0
