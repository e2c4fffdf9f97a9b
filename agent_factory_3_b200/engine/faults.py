"""Host-side fault injection for the engine's HTTP server.

Rollout clients must survive a server that drops requests, answers slowly or aborts a generation
half way (the reference's runner resumes aborted generations up to ``max_aborts`` times,
rollout/runner.py:222-249, and turns LLM errors into ``error:llm_error`` results, :214-219).
A ``FaultPlan`` makes the engine server produce exactly those failures on purpose, from the host
side only (nothing here touches a GPU):

    AF3_ENGINE_FAULTS="drop=0.1,delay_ms=50,abort_after=16,abort_rate=0.5,seed=1"

  drop         fraction of /generate requests answered 503 before they reach the engine
  delay_ms     latency added to every /generate request
  abort_after  abort a generation once it has produced this many tokens (with ``abort_rate``;
               the engine finishes it with reason {"type": "abort"}, as a pause would)
  abort_rate   fraction of generations that get the mid-generation abort
  seed         seed of the decisions (one random stream per server)
"""
from __future__ import annotations

import os
import random
from dataclasses import dataclass, fields


@dataclass
class FaultPlan:
    drop: float = 0.0
    delay_ms: float = 0.0
    abort_after: int = 0
    abort_rate: float = 0.0
    seed: int = 0

    def __post_init__(self):
        self._rng = random.Random(self.seed)
        self.dropped = 0
        self.aborted = 0

    @classmethod
    def parse(cls, spec: str) -> "FaultPlan":
        names = {f.name: f.type for f in fields(cls)}
        kw = {}
        for part in filter(None, (p.strip() for p in spec.split(","))):
            k, _, v = part.partition("=")
            if k not in names:
                raise ValueError(f"unknown fault {k!r}; known: {sorted(names)}")
            kw[k] = int(v) if k in ("abort_after", "seed") else float(v)
        return cls(**kw)

    @classmethod
    def from_env(cls) -> "FaultPlan | None":
        spec = os.environ.get("AF3_ENGINE_FAULTS")
        return cls.parse(spec) if spec else None

    # decisions (called from the server's event loop) -------------------------------------
    def should_drop(self) -> bool:
        hit = self.drop > 0 and self._rng.random() < self.drop
        self.dropped += int(hit)
        return hit

    def abort_point(self) -> int | None:
        """Token count after which this generation is aborted, or None."""
        if self.abort_after > 0 and self._rng.random() < self.abort_rate:
            return self.abort_after
        return None
