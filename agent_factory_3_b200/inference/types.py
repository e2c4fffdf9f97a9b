"""Public types of the streaming inference agent (reference: inference/types.py:22-237).

The names and fields match the reference's API so code written against its ``AgentHandle``
ports unchanged: ``AgentConfig``, ``Phase``, ``EventType``, ``EndReason``, the command
dataclasses, ``ToolReport``, ``StepInfo``, ``Event`` and ``AgentResult``.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from enum import Enum
from typing import Any, Literal, Optional, Union

from ..rollout.harmony import Conversation


@dataclass
class AgentConfig:
    """One agent against one sglang-compatible server, streaming generation."""
    server_url: str
    max_rounds: int = 10
    max_total_tokens: int = 80_000
    max_round_tokens: int = 32_000
    max_context_tokens: int = 128_000
    temperature: float = 1.0
    top_p: float = 1.0
    top_k: int = -1
    min_p: Optional[float] = None
    seed: Optional[int] = None
    tool_call_timeout: float = 60.0
    max_total_tool_time: float = 0.0          # 0 = unlimited
    auto_drop_analysis: bool = True
    harmony_custom_config_path: Optional[str] = None
    extra_round_budget: int = 4096
    extra_round_message: str = (
        "[System notice: You have run out of budget (time/rounds). Provide your final answer "
        "immediately based on what you know so far. Do not use any more tools.]")
    model_identity: str = "You are ChatGPT, a large language model trained by OpenAI."
    reasoning_effort: str = "medium"
    stream_output: bool = True                # server streams increments (else cumulative)
    http_timeout: float = 3600.0


class Phase(str, Enum):
    IDLE = "idle"
    GENERATING = "generating"
    CALLING_TOOL = "calling_tool"
    PAUSED = "paused"
    EXTRA_ROUND = "extra_round"
    DORMANT = "dormant"          # finished a run; continue_from() may start another
    COMPLETED = "completed"      # closed
    FAILED = "failed"


class EventType(str, Enum):
    STARTED = "started"
    ROUND_START = "round_start"
    STREAM_CHUNK = "stream_chunk"
    GENERATION_DONE = "generation_done"
    TOOL_CALL_START = "tool_call_start"
    TOOL_CALL_DONE = "tool_call_done"
    ROUND_DONE = "round_done"
    INJECTION_APPLIED = "injection_applied"
    PAUSED = "paused"
    RESUMED = "resumed"
    EXTRA_ROUND_START = "extra_round_start"
    COMPLETED = "completed"
    ERROR = "error"


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


DEFAULT_ASSISTANT_PREFIX = "<|channel|>final"


@dataclass(frozen=True)
class StopCommand:
    pass


@dataclass(frozen=True)
class PauseCommand:
    pass


@dataclass(frozen=True)
class ResumeCommand:
    pass


@dataclass(frozen=True)
class ForceExtraRoundCommand:
    message: Optional[str] = None      # None: AgentConfig.extra_round_message
    budget: Optional[int] = None       # None: AgentConfig.extra_round_budget
    assistant_prefix: str = DEFAULT_ASSISTANT_PREFIX


@dataclass(frozen=True)
class InjectMessageCommand:
    content: str
    role: Literal["user", "developer"] = "user"


Command = Union[StopCommand, PauseCommand, ResumeCommand, ForceExtraRoundCommand,
                InjectMessageCommand]


@dataclass
class ToolReport:
    tool_name: str
    tool_input: str
    tool_output: str
    elapsed: float
    error: Optional[str] = None        # "timeout" | "exception" | "interrupted" | None
    early_exit: bool = False


@dataclass
class StepInfo:
    type: Literal["init", "assistant", "tool"]
    round_index: int
    token_start: int
    token_end: int
    created_at: float
    elapsed: float = 0.0
    finish_reason: Optional[str] = None
    recipient: Optional[str] = None
    tool_name: Optional[str] = None
    tool_input: Optional[str] = None
    tool_output: Optional[str] = None
    tool_error: Optional[str] = None
    early_exit: bool = False


@dataclass
class AgentResult:
    end_reason: EndReason
    end_reason_detail: str
    tokens: list[int]
    conversation: Conversation
    steps: list[StepInfo]
    num_generated_tokens: int
    total_tool_time: float
    errors: list[str] = field(default_factory=list)


@dataclass
class Event:
    type: EventType
    timestamp: float
    round_index: int
    phase: Phase
    total_generated_tokens: int = 0
    chunk_tokens: Optional[list[int]] = None
    chunk_text: Optional[str] = None
    tool_name: Optional[str] = None
    tool_output: Optional[str] = None
    tool_error: Optional[str] = None
    end_reason: Optional[str] = None
    end_reason_detail: Optional[str] = None
    error: Optional[str] = None
    result: Optional[AgentResult] = None
    extra: dict[str, Any] = field(default_factory=dict)
