"""Least-busy selection among engine servers."""
from __future__ import annotations

import asyncio


class ServerPool:
    def __init__(self, urls: list[str]):
        if not urls:
            raise ValueError("ServerPool needs at least one URL")
        self.urls = list(urls)
        self.active = {u: 0 for u in self.urls}
        self._lock = asyncio.Lock()

    async def acquire(self) -> str:
        async with self._lock:
            url = min(self.urls, key=lambda u: (self.active[u], self.urls.index(u)))
            self.active[url] += 1
            return url

    async def release(self, url: str) -> None:
        async with self._lock:
            self.active[url] = max(0, self.active[url] - 1)

    def stats(self) -> dict[str, int]:
        return dict(self.active)
