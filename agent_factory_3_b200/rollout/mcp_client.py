"""Minimal async MCP client over the official ``mcp`` SDK.

A client is opened from one entry of an MCP config (``{"command", "args", "env", "cwd"}`` for a
stdio server, ``{"url"}`` for streamable HTTP) or from an in-process FastMCP server object
(tests, embedded environments).  It exposes what the tool executor needs:
``initialize_result``, ``list_tools``, ``call_tool(name, arguments, timeout)`` and ``get_prompt``.
"""
from __future__ import annotations

import asyncio
import contextlib
from datetime import timedelta
from typing import Any

from mcp import ClientSession, StdioServerParameters
from mcp.client.stdio import stdio_client


class McpClient:
    def __init__(self, spec: dict | Any):
        self.spec = spec
        self.session: ClientSession | None = None
        self.initialize_result = None
        self._stack: contextlib.AsyncExitStack | None = None

    async def __aenter__(self) -> "McpClient":
        self._stack = contextlib.AsyncExitStack()
        spec = self.spec
        if not isinstance(spec, dict):  # in-process FastMCP / lowlevel Server
            from mcp.shared.memory import create_connected_server_and_client_session

            server = getattr(spec, "_mcp_server", spec)
            self.session = await self._stack.enter_async_context(
                create_connected_server_and_client_session(server))
            self.initialize_result = getattr(self.session, "_init_result", None)
            if self.initialize_result is None:
                self.initialize_result = await self._initialize_info(server)
            return self
        if "url" in spec:
            from mcp.client.streamable_http import streamablehttp_client

            read, write, _ = await self._stack.enter_async_context(streamablehttp_client(spec["url"]))
        else:
            params = StdioServerParameters(command=spec["command"], args=list(spec.get("args", [])),
                                           env=spec.get("env"), cwd=spec.get("cwd"))
            read, write = await self._stack.enter_async_context(stdio_client(params))
        self.session = await self._stack.enter_async_context(ClientSession(read, write))
        self.initialize_result = await self.session.initialize()
        return self

    @staticmethod
    async def _initialize_info(server):
        class _Info:
            instructions = getattr(server, "instructions", None)
        return _Info()

    async def __aexit__(self, *exc):
        if self._stack is not None:
            await self._stack.aclose()
            self._stack = None

    async def list_tools(self):
        return (await self.session.list_tools()).tools

    async def call_tool(self, name: str, arguments: dict | None = None, timeout: float | None = None):
        coro = self.session.call_tool(name, arguments or {},
                                      read_timeout_seconds=timedelta(seconds=timeout) if timeout else None)
        if timeout:
            return await asyncio.wait_for(coro, timeout=timeout + 1.0)
        return await coro

    async def get_prompt(self, name: str, arguments: dict | None = None):
        return await self.session.get_prompt(name, arguments or {})
