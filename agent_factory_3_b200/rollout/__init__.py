"""Multi-turn ReAct rollouts over harmony tokens: configs, result types, LLM backends for the
sglang-compatible engine, MCP tool execution and the runner.

The package exposes the public names of the reference's rollout package
(src/agent_factory_3/rollout/__init__.py), resolved on first use so that importing one
submodule (for instance ``rollout.types`` from the trainer) does not load the MCP client or
the HTTP backends."""
from __future__ import annotations

import importlib

_EXPORTS = {
    # configs
    "ConversationConfig": ".config", "ExtraRoundConfig": ".config", "LoopConfig": ".config",
    "RecordConfig": ".config", "SamplingParams": ".config", "SegmentTemperatureConfig": ".config",
    # result types
    "EndReason": ".types", "StepType": ".types", "TruncationReason": ".types",
    "TokenBudget": ".types", "SegmentMeta": ".types", "BaseStep": ".types", "InitStep": ".types",
    "AssistantStep": ".types", "ToolStep": ".types", "Step": ".types", "ReactResult": ".types",
    "ToolErrorType": ".types",
    # tools, conversation, runner
    "McpExecutor": ".mcp_executor", "ToolCallReport": ".mcp_executor",
    "ConversationBuilder": ".conversation_builder",
    "UnifiedReactRunner": ".runner",
    # parallel execution
    "RolloutConfig": ".parallel.config", "RolloutResult": ".parallel.config",
    "execute_rollout": ".parallel.executor",
}
# the runner consumes the backends' unified completion record under this name
_ALIASES = {"CompletionResult": (".llm_backend.types", "GenerationResult")}

__all__ = sorted(list(_EXPORTS) + list(_ALIASES))


def __getattr__(name: str):
    if name in _EXPORTS:
        value = getattr(importlib.import_module(_EXPORTS[name], __name__), name)
    elif name in _ALIASES:
        mod, attr = _ALIASES[name]
        value = getattr(importlib.import_module(mod, __name__), attr)
    else:
        raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
    globals()[name] = value
    return value


def __dir__():
    return sorted(list(globals()) + __all__)
