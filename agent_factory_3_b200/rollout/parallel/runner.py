"""Stand-alone batch rollout runner (no trainer): bounded concurrency, least-busy server,
progress monitor, post-processing."""
from __future__ import annotations

import asyncio
from typing import Optional

from .backend import AsyncBackend
from .config import RolloutConfig, RolloutResult
from .execution_monitor import ExecutionMonitor
from .executor import execute_rollout
from .postprocessing import compute_stats
from .server_pool import ServerPool


class ParallelRunner:
    def __init__(self, server_urls: list[str], max_concurrency: int = 32, use_tqdm: bool = True,
                 backend_factory=None):
        self.pool = ServerPool(server_urls)
        self.backend = AsyncBackend(max_concurrency)
        self.use_tqdm = use_tqdm
        self.backend_factory = backend_factory   # url -> LLM backend (tests / in-process engines)

    async def _one(self, cfg: RolloutConfig, stop_event, monitor) -> RolloutResult:
        url = await self.pool.acquire()
        try:
            be = self.backend_factory(url) if self.backend_factory else None
            r = await execute_rollout(cfg, url, stop_event, backend=be)
        finally:
            await self.pool.release(url)
        r = compute_stats(r)
        monitor.update(r)
        return r

    async def run(self, configs: list[RolloutConfig],
                  stop_event: Optional[asyncio.Event] = None) -> list[RolloutResult]:
        mon = ExecutionMonitor(len(configs), use_tqdm=self.use_tqdm)
        try:
            return await self.backend.execute_batch(
                [lambda c=c: self._one(c, stop_event, mon) for c in configs])
        finally:
            self.summary = mon.summary()
            mon.close()

    def run_sync(self, configs: list[RolloutConfig]) -> list[RolloutResult]:
        return asyncio.run(self.run(configs))
