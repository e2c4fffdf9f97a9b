"""Streaming ReAct agent for serving and interactive inference (reference:
inference/handle.py:133-1384).

``AgentHandle`` runs one harmony-format agent against an sglang-compatible server (ours or
sglang), with MCP tools, as an asyncio task whose state can be read at any time:

* progress: ``phase``, ``round_index``, ``streaming_tokens`` / ``streaming_text`` of the
  message being generated, ``accumulated_tokens``, ``steps``, and an ``events()`` stream
  (round start, stream chunks, tool calls, injections, pause/resume, completion);
* synchronous commands, applied at safe points: ``stop()``, ``pause()`` / ``resume()`` (the
  HTTP stream is closed while paused and re-issued afterwards over prompt + partial tokens,
  which the server's prefix cache serves cheaply), ``force_extra_round()`` (interrupts
  generation or a running tool call and asks for a final answer, optionally prefilling the
  assistant turn), ``inject_message()`` (added at the next round boundary);
* ``probe()``: a side request that forks the current context (optionally including the
  partial message), asks for a final answer and returns its text without touching the
  agent's state;
* ``continue_from()``: after a run ends the handle is DORMANT and keeps its context; a new
  user (or developer) message starts another run on top of it.
"""
from __future__ import annotations

import asyncio
import contextlib
import json
import logging
import re
import time
from dataclasses import dataclass
from typing import Any, AsyncGenerator, Optional

from ..rollout.config import ConversationConfig
from ..rollout.conversation_builder import ConversationBuilder
from ..rollout.harmony import (CHANNEL, CONSTRAIN, END, MESSAGE, RETURN, CALL, START,
                               Conversation, HarmonyEncoding, Message, Role)
from ..rollout.mcp_executor import McpExecutor
from .types import (DEFAULT_ASSISTANT_PREFIX, AgentConfig, AgentResult, EndReason, Event,
                    EventType, ForceExtraRoundCommand, InjectMessageCommand, Phase, StepInfo,
                    ToolReport)

logger = logging.getLogger(__name__)

_SPECIAL_BY_NAME = {"<|start|>": START, "<|end|>": END, "<|message|>": MESSAGE,
                    "<|channel|>": CHANNEL, "<|constrain|>": CONSTRAIN, "<|return|>": RETURN,
                    "<|call|>": CALL}
_SPECIAL_RE = re.compile("(" + "|".join(re.escape(k) for k in _SPECIAL_BY_NAME) + ")")


def encode_with_specials(enc: HarmonyEncoding, text: str) -> list[int]:
    """Text in which harmony control tokens appear literally (``<|channel|>final``)."""
    ids: list[int] = []
    for part in _SPECIAL_RE.split(text):
        if not part:
            continue
        ids += [_SPECIAL_BY_NAME[part]] if part in _SPECIAL_BY_NAME else enc.tok.encode(part)
    return ids


@dataclass
class _Budget:
    max_tokens: int
    limiting: str

    @property
    def can_generate(self) -> bool:
        return self.max_tokens > 0


class _Interrupted(Exception):
    """Generation or a tool call was cut short by a command (stop / force extra round)."""


class AgentHandle:
    def __init__(self, config: AgentConfig, *, mcp_config: Optional[dict[str, Any]] = None,
                 mcp_servers: Optional[dict[str, Any]] = None,
                 encoding: Optional[HarmonyEncoding] = None):
        """``mcp_config`` is ``{"mcpServers": {name: spec}}`` (stdio command or URL);
        ``mcp_servers`` maps names to in-process FastMCP servers (embedding, tests)."""
        self._config = config
        self._mcp_config = mcp_config
        self._mcp_servers = mcp_servers or {}
        self._enc = encoding or HarmonyEncoding()
        # public state
        self._phase = Phase.IDLE
        self._round_index = 0
        self._streaming_tokens: list[int] = []
        self._committed: list[int] = []          # rendered messages (no trailing header)
        self._messages: list[Message] = []
        self._steps: list[StepInfo] = []
        self._generated = 0
        self._tool_time = 0.0
        self._errors: list[str] = []
        self._result: Optional[AgentResult] = None
        # commands (set from any coroutine of the loop; read at safe points)
        self._stop_requested = False
        self._pause_requested = False
        self._force_extra: Optional[ForceExtraRoundCommand] = None
        self._injections: list[InjectMessageCommand] = []
        self._resume_event = asyncio.Event()
        self._resume_event.set()
        self._interrupt = asyncio.Event()
        # internals
        self._events: asyncio.Queue = asyncio.Queue()
        self._task: Optional[asyncio.Task] = None
        self._executor: Optional[McpExecutor] = None
        self._session = None

    # ------------------------------------------------------------------ state
    @property
    def phase(self) -> Phase:
        return self._phase

    @property
    def round_index(self) -> int:
        return self._round_index

    @property
    def streaming_tokens(self) -> list[int]:
        return list(self._streaming_tokens)

    @property
    def streaming_text(self) -> str:
        return self._enc.decode(self._streaming_tokens)

    @property
    def accumulated_tokens(self) -> list[int]:
        return list(self._committed)

    @property
    def steps(self) -> list[StepInfo]:
        return list(self._steps)

    @property
    def total_generated_tokens(self) -> int:
        return self._generated

    @property
    def result(self) -> Optional[AgentResult]:
        return self._result

    @property
    def is_running(self) -> bool:
        return self._task is not None and not self._task.done()

    @property
    def is_alive(self) -> bool:
        return self._phase not in (Phase.COMPLETED, Phase.FAILED)

    # ------------------------------------------------------------------ commands
    def stop(self) -> None:
        """End the run at the next safe point (generation and tool calls are interrupted)."""
        self._stop_requested = True
        self._interrupt.set()
        self._resume_event.set()

    def pause(self) -> None:
        """Pause generation: the stream is closed and re-issued on resume()."""
        self._pause_requested = True
        self._resume_event.clear()

    def resume(self) -> None:
        self._pause_requested = False
        self._resume_event.set()

    def force_extra_round(self, message: Optional[str] = None, budget: Optional[int] = None,
                          assistant_prefix: str = DEFAULT_ASSISTANT_PREFIX) -> None:
        """Interrupt generation or a running tool call and ask for a final answer now.
        ``assistant_prefix`` (control tokens allowed) prefills the assistant turn."""
        self._force_extra = ForceExtraRoundCommand(message, budget, assistant_prefix)
        self._interrupt.set()
        self._resume_event.set()

    def inject_message(self, content: str, role: str = "user") -> None:
        """Queue a user/developer message; it is added at the next round boundary."""
        if role not in ("user", "developer"):
            raise ValueError("role must be 'user' or 'developer'")
        self._injections.append(InjectMessageCommand(content=content, role=role))

    # ------------------------------------------------------------------ lifecycle
    async def start(self, user_prompt: str, *, system_prompt: Optional[str] = None,
                    dev_instructions: Optional[str] = None,
                    conversation_start_date: Optional[str] = None) -> None:
        """Start the agent as a task (returns immediately).  ``system_prompt`` replaces the
        model identity line of the system message."""
        if self._task is not None:
            raise RuntimeError("agent already started")
        self._task = asyncio.create_task(self._run(user_prompt, system_prompt, dev_instructions,
                                                   conversation_start_date))

    async def events(self) -> AsyncGenerator[Event, None]:
        """Events of the current run; ends after COMPLETED or ERROR."""
        while True:
            ev = await self._events.get()
            if ev is None:
                return
            yield ev
            if ev.type in (EventType.COMPLETED, EventType.ERROR):
                return

    async def join(self) -> Optional[AgentResult]:
        if self._task is not None:
            with contextlib.suppress(Exception):
                await self._task
        return self._result

    async def continue_from(self, message: str, role: str = "user") -> None:
        """Start another run on top of the finished one (the handle must be DORMANT)."""
        if self._phase != Phase.DORMANT:
            raise RuntimeError(f"continue_from needs a DORMANT agent, not {self._phase.value}")
        self.inject_message(message, role)
        self._stop_requested = False
        self._force_extra = None
        self._interrupt.clear()
        self._events = asyncio.Queue()
        # earlier analysis messages leave the prompt once a final answer follows them
        conv = Conversation.from_messages(self._messages)
        full = self._enc.render_conversation_for_completion(conv, "assistant",
                                                            self._config.auto_drop_analysis)
        self._committed = full[:-len(self._assistant_header())]
        self._task = asyncio.create_task(self._continue_run())

    async def close(self) -> None:
        """Stop a running agent and release the MCP sessions and HTTP connections."""
        if self.is_running:
            self.stop()
            with contextlib.suppress(Exception):
                await self._task
        await self._cleanup()
        self._phase = Phase.COMPLETED

    async def probe(self, message: str = "Provide your current best answer.", budget: int = 512,
                    include_partial: bool = True, temperature: Optional[float] = None,
                    assistant_prefix: str = DEFAULT_ASSISTANT_PREFIX) -> Optional[str]:
        """Fork the current context, ask for a final answer in a separate request, return its
        text.  The running agent is not affected."""
        prompt = list(self._committed)
        if include_partial and self._streaming_tokens:
            partial = list(self._streaming_tokens)
            if partial[-1] not in (END, CALL, RETURN):
                partial.append(END)
            prompt += self._assistant_header() + partial
        prompt += self._enc.render(Message.from_role_and_content(Role.USER, message))
        prefix = encode_with_specials(self._enc, assistant_prefix)
        prompt += self._assistant_header() + prefix
        try:
            out = await self._generate_once(prompt, budget, temperature)
        except Exception as e:  # noqa: BLE001
            logger.warning("probe failed: %s", e)
            return None
        text = self._final_text(prefix + out)
        return text

    # ------------------------------------------------------------------ run
    async def _run(self, user_prompt, system_prompt, dev_instructions, start_date) -> None:
        try:
            await self._setup()
            tools = await self._executor.get_tool_configs() if self._executor.has_clients else []
            cc = ConversationConfig(model_identity=system_prompt or self._config.model_identity,
                                    reasoning_effort=self._config.reasoning_effort,
                                    dev_instructions=dev_instructions,
                                    conversation_start_date=start_date)
            conv = ConversationBuilder(cc).build(user_prompt, tools)
            self._messages = list(conv.messages)
            self._committed = self._enc.render_conversation(conv)
            self._steps.append(StepInfo("init", 0, 0, len(self._committed), time.time()))
            self._emit(EventType.STARTED)
            await self._finish_run(await self._react_loop())
        except Exception as e:  # noqa: BLE001
            logger.exception("agent run failed")
            self._fail(e)
        finally:
            self._events.put_nowait(None)

    async def _continue_run(self) -> None:
        try:
            await self._finish_run(await self._react_loop())
        except Exception as e:  # noqa: BLE001
            logger.exception("agent continuation failed")
            self._fail(e)
        finally:
            self._events.put_nowait(None)

    async def _finish_run(self, end: tuple[EndReason, str]) -> None:
        reason, detail = end
        self._result = AgentResult(end_reason=reason, end_reason_detail=detail,
                                   tokens=list(self._committed),
                                   conversation=Conversation.from_messages(list(self._messages)),
                                   steps=list(self._steps), num_generated_tokens=self._generated,
                                   total_tool_time=self._tool_time, errors=list(self._errors))
        self._phase = Phase.DORMANT
        self._emit(EventType.COMPLETED, end_reason=reason.value, end_reason_detail=detail,
                   result=self._result)

    def _fail(self, e: Exception) -> None:
        self._phase = Phase.FAILED
        self._errors.append(str(e))
        self._emit(EventType.ERROR, error=str(e))

    async def _setup(self) -> None:
        import aiohttp
        self._session = aiohttp.ClientSession(
            timeout=aiohttp.ClientTimeout(total=self._config.http_timeout))
        # MCP sessions hold anyio task groups, which must be exited by the task that entered
        # them: one owner task keeps them open until _cleanup() signals it
        self._mcp_ready, self._mcp_close = asyncio.Event(), asyncio.Event()
        self._mcp_error: Optional[BaseException] = None
        self._mcp_task = asyncio.create_task(self._mcp_owner())
        await self._mcp_ready.wait()
        if self._mcp_error is not None:
            raise self._mcp_error

    async def _mcp_owner(self) -> None:
        from ..rollout.mcp_client import McpClient
        from ..rollout.parallel.executor import setup_mcp_clients
        try:
            async with contextlib.AsyncExitStack() as stack:
                clients = await setup_mcp_clients(self._mcp_config, stack)
                for name, server in self._mcp_servers.items():
                    clients[name] = await stack.enter_async_context(McpClient(server))
                self._executor = McpExecutor(clients or None,
                                             tool_call_timeout=self._config.tool_call_timeout)
                self._mcp_ready.set()
                await self._mcp_close.wait()
        except BaseException as e:  # noqa: BLE001 - reported to _setup
            self._mcp_error = e
        finally:
            self._mcp_ready.set()

    async def _cleanup(self) -> None:
        task = getattr(self, "_mcp_task", None)
        if task is not None:
            self._mcp_close.set()
            with contextlib.suppress(BaseException):
                await task
            self._mcp_task = None
        if self._session is not None:
            with contextlib.suppress(Exception):
                await self._session.close()
            self._session = None

    def _emit(self, kind: EventType, **kw) -> None:
        self._events.put_nowait(Event(type=kind, timestamp=time.time(), round_index=self._round_index,
                                      phase=self._phase, total_generated_tokens=self._generated, **kw))

    def _assistant_header(self) -> list[int]:
        return [START] + self._enc.tok.encode("assistant")

    def _apply_injections(self) -> None:
        while self._injections:
            cmd = self._injections.pop(0)
            msg = Message.from_role_and_content(cmd.role, cmd.content)
            self._messages.append(msg)
            s = len(self._committed)
            self._committed += self._enc.render(msg)
            self._steps.append(StepInfo("init", self._round_index, s, len(self._committed), time.time()))
            self._emit(EventType.INJECTION_APPLIED, extra={"role": cmd.role, "content": cmd.content})

    def _budget(self, extra_tokens: int = 0) -> _Budget:
        c = self._config
        ctx = len(self._committed) + len(self._assistant_header()) + extra_tokens
        opts = [(c.max_round_tokens, "round"), (c.max_total_tokens - self._generated, "total"),
                (c.max_context_tokens - ctx, "context")]
        n, why = min(opts, key=lambda t: t[0])
        return _Budget(max(0, n), why)

    def _final_text(self, completion: list[int]) -> str:
        try:
            msgs = self._enc.parse_messages_from_completion_tokens(completion, role="assistant",
                                                                   strict=False)
        except Exception:  # noqa: BLE001
            msgs = []
        finals = [m for m in msgs if m.channel == "final"]
        if finals:
            return finals[-1].content.strip()
        return self._enc.decode([t for t in completion if t < 199998]).strip()

    # ------------------------------------------------------------------ react loop
    async def _react_loop(self) -> tuple[EndReason, str]:
        cfg = self._config
        end: Optional[tuple[EndReason, str]] = None
        rounds = 0
        while rounds < cfg.max_rounds:
            if self._stop_requested:
                return EndReason.INTERRUPTED, "interrupted:external_stop"
            if self._force_extra is not None:
                return await self._extra_round(EndReason.COMPLETED, "completed:forced_final")
            self._apply_injections()
            budget = self._budget()
            if not budget.can_generate:
                end = (EndReason.TOKEN_LIMIT, f"token_limit:{budget.limiting}")
                break
            self._phase = Phase.GENERATING
            self._emit(EventType.ROUND_START)
            prompt = self._committed + self._assistant_header()
            t0 = time.time()
            try:
                completion, finish = await self._generate_with_resume(prompt, budget.max_tokens)
            except _Interrupted:
                self._streaming_tokens = []
                if self._stop_requested:
                    return EndReason.INTERRUPTED, "interrupted:external_stop"
                return await self._extra_round(EndReason.COMPLETED, "completed:forced_final")
            a_start = len(self._committed)
            self._committed += self._assistant_header() + completion
            self._generated += len(completion)
            self._streaming_tokens = []
            self._emit(EventType.GENERATION_DONE, extra={"finish_reason": finish})
            try:
                parsed = self._enc.parse_messages_from_completion_tokens(completion, role="assistant")
                if not parsed:
                    raise ValueError("no message in completion")
            except Exception as e:  # noqa: BLE001
                self._errors.append(f"parse error: {e}")
                self._steps.append(StepInfo("assistant", self._round_index, a_start,
                                            len(self._committed), t0, time.time() - t0, finish))
                return EndReason.ERROR, "error:parse_error"
            self._messages += parsed
            last = parsed[-1]
            step = StepInfo("assistant", self._round_index, a_start, len(self._committed), t0,
                            time.time() - t0, finish, recipient=last.recipient)
            self._steps.append(step)
            if finish == "length":
                end = (EndReason.TOKEN_LIMIT, f"token_limit:{budget.limiting}")
                break
            if last.recipient is None:
                if last.channel == "final":
                    return EndReason.COMPLETED, "completed:final"
                self._errors.append(f"no recipient and channel {last.channel!r}: expected final")
                return EndReason.ERROR, "error:no_final_channel"
            text = (last.content or "").strip()
            if not text or last.channel == "final":
                self._errors.append(f"invalid tool call to {last.recipient}")
                return EndReason.ERROR, "error:invalid_tool_call"
            step.tool_input = text
            try:
                report = await self._call_tool(last.recipient, text)
            except _Interrupted:
                if self._stop_requested:
                    return EndReason.INTERRUPTED, "interrupted:external_stop"
                report = ToolReport(last.recipient, text, "Error: the tool call was cancelled.",
                                    0.0, error="interrupted")
                self._commit_tool(last, report, t0)
                return await self._extra_round(EndReason.COMPLETED, "completed:forced_final")
            self._commit_tool(last, report, t0)
            if report.early_exit:
                return EndReason.TOOL_EARLY_EXIT, f"tool_early_exit:{report.tool_name}"
            rounds += 1
            self._round_index += 1
            self._emit(EventType.ROUND_DONE)
        if end is None:
            end = (EndReason.MAX_ROUNDS, f"max_rounds:{cfg.max_rounds}")
        if self._stop_requested:
            return EndReason.INTERRUPTED, "interrupted:external_stop"
        return await self._extra_round(*end)

    def _commit_tool(self, call: Message, report: ToolReport, t0: float) -> None:
        msg = Message(role=call.recipient, content=report.tool_output, channel=call.channel,
                      recipient="assistant")
        self._messages.append(msg)
        s = len(self._committed)
        self._committed += self._enc.render(msg)
        self._steps.append(StepInfo("tool", self._round_index, s, len(self._committed), t0,
                                    report.elapsed, tool_name=report.tool_name,
                                    tool_input=report.tool_input, tool_output=report.tool_output,
                                    tool_error=report.error, early_exit=report.early_exit))

    async def _call_tool(self, recipient: str, text: str) -> ToolReport:
        cfg = self._config
        if cfg.max_total_tool_time > 0 and self._tool_time >= cfg.max_total_tool_time:
            return ToolReport(recipient, text, f"Error: tool time budget exceeded "
                              f"({self._tool_time:.1f}s / {cfg.max_total_tool_time:.1f}s)", 0.0,
                              error="timeout")
        self._phase = Phase.CALLING_TOOL
        self._emit(EventType.TOOL_CALL_START, tool_name=recipient)
        call = asyncio.ensure_future(self._executor.call_tool(recipient, text))
        wake = asyncio.ensure_future(self._interrupt.wait())
        done, _ = await asyncio.wait({call, wake}, return_when=asyncio.FIRST_COMPLETED)
        if call not in done:
            call.cancel()
            with contextlib.suppress(BaseException):
                await call
            raise _Interrupted()
        wake.cancel()
        r = call.result()
        self._tool_time += r.elapsed
        report = ToolReport(r.tool_name, text, r.tool_output, r.elapsed,
                            error=r.error.value if r.error is not None else None,
                            early_exit=r.early_exit)
        self._emit(EventType.TOOL_CALL_DONE, tool_name=report.tool_name,
                   tool_output=report.tool_output, tool_error=report.error)
        return report

    async def _extra_round(self, reason: EndReason, detail: str) -> tuple[EndReason, str]:
        """Ask for a final answer without tools (user notice + assistant prefill)."""
        cmd = self._force_extra or ForceExtraRoundCommand()
        forced = self._force_extra is not None
        self._force_extra = None
        self._interrupt.clear()
        cfg = self._config
        self._phase = Phase.EXTRA_ROUND
        self._emit(EventType.EXTRA_ROUND_START)
        self._apply_injections()          # queued messages precede the closing notice
        note = Message.from_role_and_content(Role.USER, cmd.message or cfg.extra_round_message)
        self._messages.append(note)
        self._committed += self._enc.render(note)
        prefix = encode_with_specials(self._enc, cmd.assistant_prefix)
        # the round exists because a budget ran out: only the context length still binds
        room = cfg.max_context_tokens - len(self._committed) - len(self._assistant_header()) - len(prefix)
        budget = min(cmd.budget or cfg.extra_round_budget, room)
        if budget <= 0:
            return reason, detail
        t0 = time.time()
        prompt = self._committed + self._assistant_header() + prefix
        try:
            out, finish = await self._generate_with_resume(prompt, budget)
        except _Interrupted:
            self._streaming_tokens = []
            return EndReason.INTERRUPTED, "interrupted:external_stop"
        completion = prefix + out
        a_start = len(self._committed)
        self._committed += self._assistant_header() + completion
        self._generated += len(out)
        self._streaming_tokens = []
        try:
            parsed = self._enc.parse_messages_from_completion_tokens(completion, role="assistant",
                                                                     strict=False)
        except Exception:  # noqa: BLE001
            parsed = []
        self._messages += parsed
        self._steps.append(StepInfo("assistant", self._round_index, a_start, len(self._committed),
                                    t0, time.time() - t0, finish))
        has_final = any(m.channel == "final" for m in parsed)
        if forced:
            return ((EndReason.COMPLETED, "completed:forced_final") if has_final
                    else (EndReason.ERROR, "error:no_final_channel"))
        return reason, f"{detail}:extra_round" if has_final else detail

    # ------------------------------------------------------------------ generation
    def _sampling(self, max_tokens: int, temperature: Optional[float] = None) -> dict:
        c = self._config
        sp = {"max_new_tokens": int(max_tokens),
              "temperature": c.temperature if temperature is None else temperature,
              "top_p": c.top_p, "top_k": c.top_k,
              "stop_token_ids": self._enc.stop_tokens_for_assistant_actions()}
        if c.min_p is not None:
            sp["min_p"] = c.min_p
        if c.seed is not None:
            sp["sampling_seed"] = c.seed
        return sp

    async def _generate_with_resume(self, prompt: list[int], max_tokens: int) -> tuple[list[int], Optional[str]]:
        """Stream one assistant turn.  pause() closes the stream; after resume() the request
        is re-issued over prompt + the tokens received so far.  stop() / force_extra_round()
        raise _Interrupted."""
        self._streaming_tokens = []
        while True:
            why, finish = await self._stream_once(prompt + self._streaming_tokens,
                                                  max_tokens - len(self._streaming_tokens))
            if why == "done":
                return list(self._streaming_tokens), finish
            if why == "interrupt" or self._stop_requested or self._force_extra is not None:
                raise _Interrupted()
            phase = self._phase
            self._phase = Phase.PAUSED
            self._emit(EventType.PAUSED)
            await self._resume_event.wait()
            if self._stop_requested or self._force_extra is not None:
                raise _Interrupted()
            self._phase = phase
            self._emit(EventType.RESUMED)
            if len(self._streaming_tokens) >= max_tokens:
                return list(self._streaming_tokens), "length"

    async def _stream_once(self, prompt: list[int], max_tokens: int) -> tuple[str, Optional[str]]:
        """One streaming request; returns ("done" | "pause" | "interrupt", finish_reason)."""
        if max_tokens <= 0:
            return "done", "length"
        body = {"input_ids": prompt, "sampling_params": self._sampling(max_tokens), "stream": True}
        finish = None
        base = len(self._streaming_tokens)   # tokens received by earlier (paused) requests
        async with self._session.post(f"{self._config.server_url}/generate", json=body) as resp:
            resp.raise_for_status()
            lines = resp.content.__aiter__()
            while True:
                if self._interrupt.is_set():
                    return "interrupt", None
                if self._pause_requested:
                    return "pause", None
                nxt = asyncio.ensure_future(lines.__anext__())
                gate = asyncio.ensure_future(self._wait_command())
                done, _ = await asyncio.wait({nxt, gate}, return_when=asyncio.FIRST_COMPLETED)
                if nxt not in done:
                    nxt.cancel()
                    with contextlib.suppress(BaseException):
                        await nxt
                    continue            # the loop head reports the command
                gate.cancel()
                try:
                    raw = nxt.result()
                except StopAsyncIteration:
                    break
                line = raw.decode().strip()
                if not line.startswith("data:"):
                    continue
                data = line[5:].strip()
                if data == "[DONE]":
                    break
                chunk = json.loads(data)
                ids = [int(t) for t in chunk.get("output_ids", [])]
                if not self._config.stream_output:      # cumulative: this request's output so far
                    ids = ids[len(self._streaming_tokens) - base:]
                if ids:
                    self._streaming_tokens += ids
                    self._emit(EventType.STREAM_CHUNK, chunk_tokens=ids,
                               chunk_text=self._enc.decode(ids))
                fr = (chunk.get("meta_info") or {}).get("finish_reason")
                if fr is not None:
                    finish = fr.get("type") if isinstance(fr, dict) else str(fr)
        return "done", finish

    async def _wait_command(self) -> None:
        """Returns when stop / force / pause is requested (polled; commands are plain calls)."""
        while not (self._interrupt.is_set() or self._pause_requested):
            await asyncio.sleep(0.01)

    async def _generate_once(self, prompt: list[int], max_tokens: int,
                             temperature: Optional[float] = None) -> list[int]:
        import aiohttp
        body = {"input_ids": prompt, "sampling_params": self._sampling(max_tokens, temperature)}
        own = self._session is None
        session = self._session or aiohttp.ClientSession(
            timeout=aiohttp.ClientTimeout(total=self._config.http_timeout))
        try:
            async with session.post(f"{self._config.server_url}/generate", json=body) as resp:
                resp.raise_for_status()
                out = await resp.json()
        finally:
            if own:
                await session.close()
        return [int(t) for t in out.get("output_ids", [])]
