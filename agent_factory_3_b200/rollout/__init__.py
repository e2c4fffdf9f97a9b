"""Multi-turn ReAct rollouts over harmony tokens: configs, result types, LLM backends for the
sglang-compatible engine, MCP tool execution and the runner."""
