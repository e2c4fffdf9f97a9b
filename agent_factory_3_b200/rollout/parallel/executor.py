"""One rollout end to end: spawn the MCP clients (cross-process rate limited), discover tools,
build the conversation, run the ReAct loop against one engine URL, always return a
RolloutResult (reference: rollout/parallel/executor.py:77-383).  ``MCP_DEBUG=1`` logs client
lifecycle with open-fd and child-process counts (to ``MCP_DEBUG_LOG`` when set)."""
from __future__ import annotations

import asyncio
import contextlib
import os
import time
import traceback
from typing import Any, Optional

from ..config import LoopConfig
from ..conversation_builder import ConversationBuilder
from ..harmony import START, Conversation, HarmonyEncoding
from ..llm_backend.sglang_backend import SGLangBackend
from ..mcp_client import McpClient
from ..mcp_executor import McpExecutor
from ..runner import UnifiedReactRunner
from .config import RolloutConfig, RolloutResult

_MCP_DEBUG = os.environ.get("MCP_DEBUG") == "1"


def _count_fds() -> int:
    try:
        return len(os.listdir("/proc/self/fd"))
    except OSError:
        return -1


def _count_children() -> int:
    try:
        import psutil
        return len(psutil.Process().children(recursive=True))
    except Exception:  # noqa: BLE001
        return -1


def mcp_debug(rid: str, msg: str) -> None:
    if not _MCP_DEBUG:
        return
    line = f"[MCP_DEBUG] {time.time():.3f} pid={os.getpid()} [{rid}] {msg}\n"
    path = os.environ.get("MCP_DEBUG_LOG")
    if path:
        with open(path, "a") as f:
            f.write(line)
    else:
        print(line, end="", flush=True)


class CrossProcessSpawnLimiter:
    """At most one MCP server spawn every ``min_interval`` seconds across all processes of
    this user (an flock'ed timestamp file)."""

    def __init__(self, min_interval: float = 0.25, lock_path: str | None = None):
        self.min_interval = min_interval
        self.lock_path = lock_path or f"/tmp/.af3_mcp_spawn_{os.getuid()}.lock"

    def _gate(self):
        import fcntl
        fd = os.open(self.lock_path, os.O_CREAT | os.O_RDWR, 0o666)
        try:
            fcntl.flock(fd, fcntl.LOCK_EX)
            try:
                os.lseek(fd, 0, os.SEEK_SET)
                data = os.read(fd, 32)
                last = float(data) if data else 0.0
            except (ValueError, OSError):
                last = 0.0
            wait = last + self.min_interval - time.time()
            if wait > 0:
                time.sleep(wait)
            os.lseek(fd, 0, os.SEEK_SET)
            os.ftruncate(fd, 0)
            os.write(fd, str(time.time()).encode())
            fcntl.flock(fd, fcntl.LOCK_UN)
        finally:
            os.close(fd)

    async def __aenter__(self):
        await asyncio.get_running_loop().run_in_executor(None, self._gate)
        return self

    async def __aexit__(self, *exc):
        return False


_LIMITER: CrossProcessSpawnLimiter | None = None


def description_overrides(mcp_config: Optional[dict]) -> dict:
    out = {}
    for key, sc in ((mcp_config or {}).get("mcpServers") or {}).items():
        if not isinstance(sc, dict):
            continue
        td, io = sc.get("toolDescriptions"), sc.get("instructionsOverride")
        if td is not None or io is not None:
            out[key] = {"instructions": io, "tools": td or {}}
    return out


async def setup_mcp_clients(mcp_config: Optional[dict], stack: contextlib.AsyncExitStack, *,
                            spawn_interval: float = 0.0, rollout_id: str = "") -> dict[str, Any]:
    global _LIMITER
    clients = {}
    for key, sc in ((mcp_config or {}).get("mcpServers") or {}).items():
        client = McpClient(sc)
        mcp_debug(rollout_id, f"client_enter key={key}")
        if spawn_interval > 0:
            if _LIMITER is None:
                _LIMITER = CrossProcessSpawnLimiter(spawn_interval)
            async with _LIMITER:
                await stack.enter_async_context(client)
        else:
            await stack.enter_async_context(client)
        clients[key] = client
        mcp_debug(rollout_id, f"client_ready key={key} fds={_count_fds()} children={_count_children()}")
    return clients


def create_backend(loop: LoopConfig, server_url: str, cache_salt: Optional[str] = None):
    return SGLangBackend(server_url, num_layers=loop.num_hidden_layers,
                         num_experts_per_tok=loop.num_experts_per_tok,
                         lora_path=loop.lora_adapter_name, cache_salt=cache_salt)


def make_result(config: RolloutConfig, start: float, server_url: str, result=None,
                error: Exception | None = None) -> RolloutResult:
    end = time.time()
    return RolloutResult(rollout_id=config.rollout_id, result=result, start_time=start,
                         end_time=end, elapsed_time=end - start, server_url=server_url,
                         success=error is None and result is not None,
                         error=None if error is None else f"{type(error).__name__}: {error}",
                         traceback=None if error is None else traceback.format_exc())


async def execute_rollout(config: RolloutConfig, server_url: str,
                          stop_event: Optional[asyncio.Event] = None, *,
                          base_conversation: Optional[Conversation] = None,
                          base_tokens: Optional[list[int]] = None,
                          backend=None, encoding: HarmonyEncoding | None = None) -> RolloutResult:
    """Run one rollout; ``backend`` overrides the HTTP client (tests / in-process engines)."""
    start = time.time()
    rid = config.rollout_id
    if base_tokens is not None and base_conversation is None:
        raise ValueError("base_tokens requires base_conversation")
    out = None
    try:
        async with contextlib.AsyncExitStack() as stack:
            clients = await setup_mcp_clients(config.mcp_config, stack,
                                              spawn_interval=config.loop_config.mcp_spawn_interval,
                                              rollout_id=rid)
            ex = McpExecutor(clients or None, tool_call_timeout=config.loop_config.tool_call_timeout,
                             filter_by_include_in_prompt=config.loop_config.filter_by_include_in_prompt,
                             description_overrides=description_overrides(config.mcp_config))
            tool_configs = await ex.get_tool_configs()
            builder = ConversationBuilder(config.conv_config)
            be = backend or create_backend(config.loop_config, server_url, config.loop_config.cache_salt)
            try:
                runner = UnifiedReactRunner(be, ex, config.loop_config, encoding)
                prompt = await ex.resolve_prompts(config.user_prompt)
                initial = None
                if base_conversation is not None:
                    conv = builder.append_user_message(base_conversation, prompt)
                    if base_tokens is not None:
                        um = conv.messages[-1]
                        initial = list(base_tokens) + runner.encoding.render(um) + [START] + \
                            runner.encoding.tok.encode("assistant")
                else:
                    conv = builder.build(prompt, tool_configs)
                res = await runner.run(conv, initial_tokens=initial, stop_event=stop_event,
                                       record_config=config.record_config, rollout_id=rid)
                out = make_result(config, start, server_url, result=res)
            finally:
                if backend is None:
                    await be.close()
    except Exception as e:  # noqa: BLE001
        if out is not None:  # MCP teardown failed after a finished rollout: keep the data
            return out
        return make_result(config, start, server_url, error=e)
    return out
