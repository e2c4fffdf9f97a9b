"""Packed-batch collation and the deterministic, cost-balanced packed sampler."""
