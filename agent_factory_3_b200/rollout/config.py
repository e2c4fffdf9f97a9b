"""Rollout configuration (field names and validation rules of the reference's
rollout/config.py:8-216)."""
from __future__ import annotations

from typing import Literal, Optional

from pydantic import BaseModel, Field, model_validator


class SamplingParams(BaseModel):
    temperature: float = 1.0
    top_p: float = 1.0
    top_k: int = -1
    min_p: Optional[float] = None
    seed: Optional[int] = None


class ConversationConfig(BaseModel):
    model_identity: str = "You are ChatGPT, a large language model trained by OpenAI."
    conversation_start_date: Optional[str] = None
    reasoning_effort: str = "medium"
    dev_instructions: Optional[str] = None


class SegmentTemperatureConfig(BaseModel):
    """Two-phase sampling: header tokens (up to <|message|>) with ``header_temperature``, the
    content with a per-recipient, per-channel or default temperature (in that priority)."""
    header_temperature: float = Field(default=0.3, ge=0.0, le=2.0)
    default_content_temperature: float = Field(default=1.0, ge=0.0, le=2.0)
    channel_temperatures: dict[str, float] = Field(default_factory=dict)
    recipient_temperatures: dict[str, float] = Field(default_factory=dict)

    def get_content_temperature(self, channel: Optional[str], recipient: Optional[str]) -> float:
        if recipient and recipient in self.recipient_temperatures:
            return self.recipient_temperatures[recipient]
        if channel and channel in self.channel_temperatures:
            return self.channel_temperatures[channel]
        return self.default_content_temperature


class ExtraRoundConfig(BaseModel):
    """Forced final answer when a rollout ends on TOKEN_LIMIT or MAX_ROUNDS."""
    budget: int = Field(default=4096, gt=0)
    message: str = ("[System notice: You have run out of budget (time/rounds). Provide your final "
                    "answer immediately based on what you know so far. Do not use any more tools.]")
    min_budget: int = Field(default=64, ge=0)
    on_token_limit: bool = True
    on_max_rounds: bool = True

    @model_validator(mode="after")
    def _validate(self):
        if self.min_budget > self.budget:
            raise ValueError(f"extra round: the token floor min_budget={self.min_budget} is "
                             f"above the budget {self.budget}")
        if not (self.on_token_limit or self.on_max_rounds):
            raise ValueError("extra round enabled with no trigger: set on_token_limit or "
                             "on_max_rounds")
        return self


class LoopConfig(BaseModel):
    backend: Literal["vllm", "sglang"] = "sglang"
    model_name: Optional[str] = None
    sampling: SamplingParams = Field(default_factory=SamplingParams)
    num_hidden_layers: Optional[int] = None
    num_experts_per_tok: Optional[int] = None
    max_rounds: int = 10
    max_total_tokens: int = 80_000
    max_round_tokens: int = 32_000
    max_context_tokens: int = 128_000
    tool_call_timeout: float = 60.0
    max_total_tool_time: float = 0.0
    tool_error_strategy: Literal["continue", "stop"] = "continue"
    filter_by_include_in_prompt: bool = True
    auto_drop_analysis: bool = True
    harmony_custom_config_path: Optional[str] = None
    max_parse_retries: int = 0
    use_streaming: bool = True
    max_aborts: int = 20
    cache_salt: Optional[str] = None
    lora_adapter_name: Optional[str] = None
    mcp_spawn_interval: float = 0.0
    segment_temperature: Optional[SegmentTemperatureConfig] = None
    extra_round: Optional[ExtraRoundConfig] = None

    @model_validator(mode="after")
    def _check_parse_retry_abort_mutual_exclusion(self):
        # a parse retry rolls the conversation back to before the failed turn, which would
        # drop the partial output an abort/resume keeps; the two recovery paths cannot mix
        if self.max_parse_retries > 0 and self.max_aborts > 0:
            raise ValueError(f"choose one recovery path: max_parse_retries={self.max_parse_retries} "
                             f"and max_aborts={self.max_aborts} are both enabled, but a parse-retry "
                             f"rollback would discard an aborted turn's partial output")
        return self

    @model_validator(mode="after")
    def _check_backend_supported(self):
        if self.backend == "vllm":
            raise NotImplementedError("backend='vllm' is not supported for training rollouts; "
                                      "use backend='sglang' (the built-in engine speaks its API)")
        return self


class RecordConfig(BaseModel):
    logprobs: bool = True
    top_logprobs: int = 0
    routing_indices: bool = False
    usage: bool = True
    entropy: bool = False
