"""Rollout result types (reference: rollout/types.py:29-443).

``ReactResult`` keeps the full token sequence of a multi-turn episode with per-token
log-probs, entropies, top-k log-probs and MoE routing ids, the step index (init / assistant /
tool) and the parsed conversation.  Serialisation is compact: routing as base64 uint8
[T, L, K] with 255 marking tokens that never went through a forward pass (prefix-cache hits),
log-probs and entropies as base64 float16 with NaN for missing values.
"""
from __future__ import annotations

import base64
from dataclasses import dataclass
from enum import Enum
from typing import Annotated, Any, Literal, Optional, Union

import numpy as np
from pydantic import BaseModel, ConfigDict, Field, field_serializer, field_validator

from .harmony import Conversation, HarmonyEncoding


class EndReason(str, Enum):
    COMPLETED = "completed"
    TOOL_EARLY_EXIT = "tool_early_exit"
    MAX_ROUNDS = "max_rounds"
    TOKEN_LIMIT = "token_limit"
    INTERRUPTED = "interrupted"
    ERROR = "error"

    @property
    def is_success(self) -> bool:
        return self in (EndReason.COMPLETED, EndReason.TOOL_EARLY_EXIT, EndReason.MAX_ROUNDS)


class StepType(str, Enum):
    INIT = "init"
    ASSISTANT = "assistant"
    TOOL = "tool"


class TruncationReason(str, Enum):
    ROUND_LIMIT = "round_limit"
    CONTEXT_SPACE = "context_space"
    GENERATION_QUOTA = "generation_quota"


class ToolErrorType(str, Enum):
    TIMEOUT = "timeout"
    EXCEPTION = "exception"
    NOT_FOUND = "not_found"
    INVALID_ARGS = "invalid_args"
    TOOL_ERROR = "tool_error"
    BUDGET_EXCEEDED = "budget_exceeded"


@dataclass
class TokenBudget:
    max_tokens: int
    limiting_factor: TruncationReason

    @property
    def can_generate(self) -> bool:
        return self.max_tokens > 0


class SegmentMeta(BaseModel):
    phase: Literal["header", "content"]
    start: int
    end: int
    temperature: float
    channel: Optional[str] = None
    recipient: Optional[str] = None


class WeightSegment(BaseModel):
    """Tokens of one assistant step produced by one weight version (abort/resume across a
    weight update splits a step into several segments); offsets relative to the step start."""
    start: int
    end: int
    weight_version: str


class AbortRecord(BaseModel):
    round_index: int
    weight_version: Optional[str]
    partial_token_count: int
    timestamp: float


class BaseStep(BaseModel):
    type: StepType
    start: int
    end: int
    round_index: Optional[int] = None
    message_start: Optional[int] = None
    message_end: Optional[int] = None
    created_at: Optional[float] = None
    elapsed: Optional[float] = None

    @property
    def length(self) -> int:
        return self.end - self.start

    @property
    def message_count(self) -> int:
        if self.message_start is None or self.message_end is None:
            return 0
        return self.message_end - self.message_start


class InitStep(BaseStep):
    type: Literal[StepType.INIT] = StepType.INIT
    num_system_tokens: Optional[int] = None
    num_developer_tokens: Optional[int] = None
    num_user_tokens: Optional[int] = None


class AssistantStep(BaseStep):
    type: Literal[StepType.ASSISTANT] = StepType.ASSISTANT
    stop_reason: Optional[str] = None
    truncation_reason: Optional[TruncationReason] = None
    recipient: Optional[str] = None
    tool_input: Optional[str] = None
    usage: Optional[dict[str, Any]] = None
    segments: list[SegmentMeta] = Field(default_factory=list)
    weight_segments: list[WeightSegment] = Field(default_factory=list)
    parse_error: Optional[str] = None


class ToolStep(BaseStep):
    type: Literal[StepType.TOOL] = StepType.TOOL
    tool_name: str
    tool_input: str
    tool_output: str
    error: Optional[ToolErrorType] = None
    early_exit: bool = False
    structured_output: Optional[dict[str, Any]] = None


Step = Annotated[Union[InitStep, AssistantStep, ToolStep], Field(discriminator="type")]


def _f16_encode(v):
    if v is None:
        return None
    arr = np.array([np.nan if x is None else x for x in v], dtype=np.float16)
    return {"dtype": "float16", "data": base64.b64encode(arr.tobytes()).decode()}


def _f16_decode(v):
    if isinstance(v, dict) and "data" in v:
        arr = np.frombuffer(base64.b64decode(v["data"]), dtype=np.float16)
        return [None if np.isnan(x) else float(x) for x in arr]
    return v


class ReactResult(BaseModel):
    model_config = ConfigDict(arbitrary_types_allowed=True)

    end_reason: EndReason
    end_reason_detail: str
    errors: list[str] = Field(default_factory=list)
    tokens: list[int]
    logprobs: Optional[list[Optional[float]]] = None
    entropy: Optional[list[Optional[float]]] = None
    top_logprobs: Optional[list[Optional[dict[int, float]]]] = None
    routing_indices: Optional[list[Optional[Any]]] = None
    steps: list[Step]
    conversation: Conversation
    total_tool_time: float
    num_generated_tokens: int
    abort_records: list[AbortRecord] = Field(default_factory=list)

    # ---- serde ----
    @field_serializer("routing_indices")
    def _ser_routing(self, v):
        if v is None:
            return None
        sample = next((x for x in v if x is not None), None)
        if sample is None:
            return None
        s = np.asarray(sample)
        arr = np.full((len(v), s.shape[0], s.shape[1]), 255, dtype=np.uint8)
        for i, ri in enumerate(v):
            if ri is not None:
                arr[i] = np.asarray(ri, dtype=np.uint8)
        return {"shape": list(arr.shape), "dtype": "uint8", "sentinel": 255,
                "data": base64.b64encode(arr.tobytes()).decode()}

    @field_validator("routing_indices", mode="before")
    @classmethod
    def _de_routing(cls, v):
        if isinstance(v, dict) and "data" in v:
            arr = np.frombuffer(base64.b64decode(v["data"]), dtype=np.uint8).reshape(v["shape"])
            sent = v.get("sentinel", 255)
            return [None if row[0, 0] == sent else row.copy() for row in arr]
        return v

    @field_serializer("logprobs")
    def _ser_lp(self, v):
        return _f16_encode(v)

    @field_validator("logprobs", mode="before")
    @classmethod
    def _de_lp(cls, v):
        return _f16_decode(v)

    @field_serializer("entropy")
    def _ser_ent(self, v):
        return _f16_encode(v)

    @field_validator("entropy", mode="before")
    @classmethod
    def _de_ent(cls, v):
        return _f16_decode(v)

    @field_serializer("conversation")
    def _ser_conv(self, c: Conversation):
        return c.to_dict()

    @field_validator("conversation", mode="before")
    @classmethod
    def _de_conv(cls, v):
        return Conversation.from_dict(v) if isinstance(v, dict) else v

    # ---- queries ----
    @property
    def is_success(self) -> bool:
        return self.end_reason.is_success

    @property
    def has_tool_errors(self) -> bool:
        return any(isinstance(s, ToolStep) and s.error is not None for s in self.steps)

    @property
    def tool_error_count(self) -> int:
        return sum(1 for s in self.steps if isinstance(s, ToolStep) and s.error is not None)

    def get_step_tokens(self, step: BaseStep) -> list[int]:
        return self.tokens[step.start:step.end]

    def get_step_text(self, step: BaseStep, encoding: HarmonyEncoding | None = None) -> str:
        return (encoding or HarmonyEncoding()).decode(self.tokens[step.start:step.end])

    def get_step_logprobs(self, step: BaseStep):
        return None if self.logprobs is None else self.logprobs[step.start:step.end]

    def get_step_routing(self, step: BaseStep):
        return None if self.routing_indices is None else self.routing_indices[step.start:step.end]

    def get_step_messages(self, step: BaseStep) -> list:
        if step.message_start is None or step.message_end is None:
            return []
        return list(self.conversation.messages[step.message_start:step.message_end])

    def get_assistant_steps(self) -> list[AssistantStep]:
        return [s for s in self.steps if s.type == StepType.ASSISTANT]

    def get_tool_steps(self) -> list[ToolStep]:
        return [s for s in self.steps if s.type == StepType.TOOL]

    def get_loss_mask(self) -> list[bool]:
        mask = [False] * len(self.tokens)
        for s in self.steps:
            if s.type == StepType.ASSISTANT:
                for i in range(s.start, s.end):
                    mask[i] = True
        return mask

    def get_trainable_data(self, logprob_fill_value: float = 0.0):
        mask = self.get_loss_mask()
        lps = [logprob_fill_value if (self.logprobs is None or self.logprobs[i] is None)
               else self.logprobs[i] for i in range(len(self.tokens))]
        return list(self.tokens), lps, mask
