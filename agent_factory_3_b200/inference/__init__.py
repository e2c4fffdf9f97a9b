"""Streaming inference agent (``AgentHandle``) and its public types."""
from .handle import AgentHandle, encode_with_specials
from .types import (DEFAULT_ASSISTANT_PREFIX, AgentConfig, AgentResult, Command, EndReason, Event,
                    EventType, ForceExtraRoundCommand, InjectMessageCommand, PauseCommand, Phase,
                    ResumeCommand, StepInfo, StopCommand, ToolReport)

__all__ = ["AgentHandle", "AgentConfig", "AgentResult", "Command", "DEFAULT_ASSISTANT_PREFIX",
           "EndReason", "Event", "EventType", "ForceExtraRoundCommand", "InjectMessageCommand",
           "PauseCommand", "Phase", "ResumeCommand", "StepInfo", "StopCommand", "ToolReport",
           "encode_with_specials"]
