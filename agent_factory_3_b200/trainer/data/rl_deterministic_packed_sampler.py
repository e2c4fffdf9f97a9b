"""Module path of the reference's packed sampler (trainer/data/rl_deterministic_packed_sampler.py);
the implementation is ``trainer.data.sampler``."""
from .sampler import (DeterministicPackedBatchSampler, PackingStats, SampleInfo,
                      pack_samples_into_bucket_groups)

__all__ = ["DeterministicPackedBatchSampler", "PackingStats", "SampleInfo",
           "pack_samples_into_bucket_groups"]
