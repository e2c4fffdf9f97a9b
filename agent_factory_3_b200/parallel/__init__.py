"""Multi-GPU plumbing: process groups, the rank-0-driven RPC control plane, NVLink symmetric
memory and the fused compute+collective paths."""
