"""Semaphore-bounded async execution of rollout tasks (batch and as-completed streaming)."""
from __future__ import annotations

import asyncio
from typing import AsyncIterator, Awaitable, Callable, Generic, TypeVar

T = TypeVar("T")
Task = Callable[[], Awaitable[T]]


class AsyncBackend(Generic[T]):
    def __init__(self, max_concurrency: int = 20):
        if max_concurrency <= 0:
            raise ValueError("max_concurrency must be positive")
        self.max_concurrency = max_concurrency

    async def execute_batch(self, tasks: list[Task]) -> list:
        sem = asyncio.Semaphore(self.max_concurrency)

        async def run(t):
            async with sem:
                return await t()

        return list(await asyncio.gather(*(run(t) for t in tasks))) if tasks else []

    async def execute_batch_streaming(self, tasks: list[Task]) -> AsyncIterator[tuple[int, T]]:
        sem = asyncio.Semaphore(self.max_concurrency)

        async def run(t, i):
            async with sem:
                return i, await t()

        pending = {asyncio.create_task(run(t, i)) for i, t in enumerate(tasks)}
        while pending:
            done, pending = await asyncio.wait(pending, return_when=asyncio.FIRST_COMPLETED)
            for d in done:
                yield d.result()
