"""agent_factory_3_b200 — a Blackwell (B200, sm_100a) native async agentic-RL framework for
gpt-oss: MXFP4-aware LoRA training with routing replay and DDIS, an sglang-compatible rollout
engine, MCP tool environments and the orchestration that ties them together.

The GPU hot paths are hand-written sm_100a kernels (tcgen05 + TMEM + TMA) in the in-tree
extension ``agent_factory_3_b200._C``; everything else is PyTorch and Python.
"""

__version__ = "0.1.0"
