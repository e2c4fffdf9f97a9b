"""MCP tool environments (each module is an MCP server: ``python -m
agent_factory_3_b200.envs.<name> ...``) and their pure game logic for in-process use."""
