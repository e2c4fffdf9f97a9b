"""Deterministic packing of a step's samples into per-rank buckets (reference:
trainer/data/rl_deterministic_packed_sampler.py:97-310).

Samples are sorted by (length desc, index asc) and each goes to the least-loaded bucket that
still fits under ``max_capacity`` tokens; a new group of ``world_size`` buckets opens when none
fits.  Empty buckets are filled from the heaviest donor, buckets are ordered by load and
grouped ``world_size`` at a time, and odd groups are reversed (zig-zag) so rank 0 is not always
the heaviest.

"Load" is a bucket's token count (the reference's rule, ``balance="tokens"``) or its estimated
compute cost (``balance="cost"``).  A packed sequence's attention work grows with the square of
each sample's length while everything else grows linearly, so two buckets with equal token
counts can differ in step time by the ratio of their sums of squared lengths, and every
data-parallel rank waits for the slowest one at the gradient reduction.  The cost of a sample of
n tokens is modelled as ``n + n^2 / attention_tokens``: ``attention_tokens`` is the length at
which a sample's causal-attention time equals the time of its linear work (projections, MoE,
loss).  The capacity limit always counts tokens.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class SampleInfo:
    index: int
    length: int


@dataclass
class PackingStats:
    num_samples: int
    num_buckets: int
    num_groups: int
    avg_bucket_load: float
    max_bucket_load: int
    min_bucket_load: int
    utilization_rate: float


def sample_cost(length: int, attention_tokens: float | None) -> float:
    """Estimated compute cost of one sample (token units); plain length without a model."""
    if not attention_tokens:
        return float(length)
    return length + length * length / float(attention_tokens)


def pack_samples_into_bucket_groups(samples: list[SampleInfo], *, max_capacity: int,
                                    world_size: int, attention_tokens: float | None = None):
    if world_size <= 0:
        raise ValueError(f"world_size must be positive, got {world_size}")
    if max_capacity <= 0:
        raise ValueError(f"max_capacity must be positive, got {max_capacity}")
    if len(samples) < world_size:
        raise RuntimeError(f"Need at least world_size samples ({world_size}), got {len(samples)}")
    for s in samples:
        if s.length > max_capacity:
            raise ValueError(f"Sample {s.index} length {s.length} exceeds max_capacity {max_capacity}.")
    cost = {s.index: sample_cost(s.length, attention_tokens) for s in samples}
    order = sorted(samples, key=lambda s: (-s.length, s.index))
    buckets: list[list[SampleInfo]] = [[] for _ in range(world_size)]
    loads = [0] * world_size          # tokens (capacity)
    work = [0.0] * world_size         # balancing load: tokens, or estimated cost
    for s in order:
        best = -1
        for i, ld in enumerate(loads):
            if ld + s.length <= max_capacity and (best < 0 or work[i] < work[best]):
                best = i
        if best < 0:
            buckets.extend([] for _ in range(world_size))
            loads.extend([0] * world_size)
            work.extend([0.0] * world_size)
            best = len(loads) - world_size
        buckets[best].append(s)
        loads[best] += s.length
        work[best] += cost[s.index]
    # fill empty buckets from the heaviest donor with more than one sample
    for e in [i for i, b in enumerate(buckets) if not b]:
        placed = False
        for d in sorted((i for i, b in enumerate(buckets) if b), key=lambda i: (-work[i], i)):
            if len(buckets[d]) <= 1:
                continue
            for c in sorted(buckets[d], key=lambda s: (s.length, s.index)):
                if loads[e] + c.length <= max_capacity:
                    buckets[d].remove(c)
                    loads[d] -= c.length
                    work[d] -= cost[c.index]
                    buckets[e].append(c)
                    loads[e] += c.length
                    work[e] += cost[c.index]
                    placed = True
                    break
            if placed:
                break
        if not placed:
            raise RuntimeError(f"Unable to redistribute to fill empty bucket #{e}; reduce "
                               f"world_size or raise max_capacity ({max_capacity}).")
    triples = sorted(zip(buckets, loads, work), key=lambda x: (-x[2], [s.index for s in x[0]]))
    ob = [b for b, _, _ in triples]
    ol = [l for _, l, _ in triples]
    groups = [ob[i:i + world_size] for i in range(0, len(ob), world_size)]
    total = sum(ol)
    stats = PackingStats(len(samples), len(ob), len(groups), total / len(ob), max(ol), min(ol),
                         total / (len(ob) * max_capacity))
    return groups, stats


class DeterministicPackedBatchSampler:
    """Yields, per bucket, the sample indices of that bucket; bucket k of group g goes to rank
    k (after zig-zag).  ``plan_for_rank(r)`` gives rank r's microbatches."""

    def __init__(self, lengths: list[int], *, max_capacity: int, world_size: int,
                 balance_ranks: bool = True, balance: str = "tokens",
                 attention_tokens: float | None = None):
        if balance not in ("tokens", "cost"):
            raise ValueError(f"balance must be 'tokens' or 'cost', got {balance!r}")
        self.world_size = world_size
        groups, self.stats = pack_samples_into_bucket_groups(
            [SampleInfo(i, int(n)) for i, n in enumerate(lengths)], max_capacity=max_capacity,
            world_size=world_size,
            attention_tokens=attention_tokens if balance == "cost" else None)
        plan = []
        for gi, group in enumerate(groups):
            if balance_ranks and gi % 2 == 1:
                group = list(reversed(group))
            plan.extend([s.index for s in b] for b in group)
        self.plan = plan

    def __iter__(self):
        yield from self.plan

    def __len__(self):
        return len(self.plan)

    def plan_for_rank(self, rank: int) -> list[list[int]]:
        return self.plan[rank::self.world_size]
