"""Run an engine's HTTP server on a background thread (in-process deployments and tests)."""
from __future__ import annotations

import asyncio
import socket
import threading

from aiohttp import web

from .scheduler import Engine
from .server import build_app


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class LocalEngineServer:
    def __init__(self, engine: Engine, host: str = "127.0.0.1", port: int | None = None):
        self.engine = engine
        self.host = host
        self.port = port or free_port()
        self._loop = None
        self._runner = None
        self._thread = None
        self._ready = threading.Event()

    @property
    def url(self) -> str:
        return f"http://{self.host}:{self.port}"

    def start(self) -> "LocalEngineServer":
        def run():
            self._loop = asyncio.new_event_loop()
            asyncio.set_event_loop(self._loop)
            self._runner = web.AppRunner(build_app(self.engine))
            self._loop.run_until_complete(self._runner.setup())
            site = web.TCPSite(self._runner, self.host, self.port)
            self._loop.run_until_complete(site.start())
            self._ready.set()
            self._loop.run_forever()

        self._thread = threading.Thread(target=run, daemon=True, name="af3-engine-http")
        self._thread.start()
        if not self._ready.wait(30):
            raise RuntimeError("engine HTTP server did not start")
        return self

    def stop(self) -> None:
        if self._loop is not None:
            fut = asyncio.run_coroutine_threadsafe(self._runner.cleanup(), self._loop)
            try:
                fut.result(10)
            except Exception:  # noqa: BLE001
                pass
            self._loop.call_soon_threadsafe(self._loop.stop)
        if self._thread is not None:
            self._thread.join(timeout=10)
        self.engine.stop()
