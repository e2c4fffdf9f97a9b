"""Module path of the reference's routing-replay activator (models/gpt_oss/routing_replay.py).
Replay is native to ``GptOssForCausalLM.forward_hidden(routing_indices=...)``."""
from .compat import enable_routing_replay

__all__ = ["enable_routing_replay"]
