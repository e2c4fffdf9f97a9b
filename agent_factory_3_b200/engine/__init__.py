"""Rollout inference engine: paged KV cache with prefix caching, continuous batching,
pause/abort/continue, LoRA serving, weight versions and routed-expert capture behind an
sglang-compatible HTTP API (``python -m agent_factory_3_b200.engine.server``)."""
