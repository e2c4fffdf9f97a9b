"""Multi-turn ReAct loop over harmony tokens (reference: rollout/runner.py:79-1166).

Per round: token budget -> generate -> (abort: keep the partial tokens, record a
WeightSegment and an AbortRecord, re-issue; the engine holds the request until generation
continues) -> accumulate log-probs / entropy / top-k / routing (routing returned for the whole
prompt overwrites the prefix positions, which covers prefix-cache hits) -> harmony parse
(optional retry with rollback) -> classify the last message: final answer, empty tool call,
tool call in the final channel, or tool call -> MCP tool call under the total tool-time budget
-> render the tool message -> early exit / error strategy.  After the loop an optional
"extra round" injects a notice and forces a final answer when the episode ended on the token
or round limit.  Segment-aware temperature samples the header (up to <|message|>) and the
content with different temperatures.
"""
from __future__ import annotations

import asyncio
import logging
import time
from typing import Optional

from .config import LoopConfig, RecordConfig
from .harmony import (CHANNEL, MESSAGE, START, Conversation, HarmonyEncoding, Message, Role,
                      StreamableParser)
from .llm_backend.protocol import LLMBackend
from .llm_backend.types import GenerationResult
from .mcp_executor import McpExecutor, ToolCallReport
from .types import (AbortRecord, AssistantStep, EndReason, InitStep, ReactResult, SegmentMeta,
                    TokenBudget, ToolErrorType, ToolStep, TruncationReason, WeightSegment)

logger = logging.getLogger(__name__)

_LIMIT_DETAIL = {
    TruncationReason.ROUND_LIMIT: "token_limit:round_limit",
    TruncationReason.CONTEXT_SPACE: "token_limit:context_space",
    TruncationReason.GENERATION_QUOTA: "token_limit:generation_quota",
}


class _Acc:
    """Per-token accumulators kept aligned with the token list."""

    def __init__(self, n: int, record: Optional[RecordConfig]):
        self.tokens: list[int] = []
        self.logprobs = [None] * n if record and record.logprobs else None
        self.top = [None] * n if record and record.top_logprobs > 0 else None
        self.entropy = [None] * n if record and record.entropy else None
        self.routing = [None] * n if record and record.routing_indices else None

    def pad(self, n: int):
        for a in (self.logprobs, self.top, self.entropy, self.routing):
            if a is not None:
                a.extend([None] * n)

    def add_completion(self, c: GenerationResult, prompt_len: int):
        n = len(c.token_ids)
        if self.logprobs is not None:
            self.logprobs.extend(c.logprobs if c.logprobs is not None else [None] * n)
        if self.top is not None:
            self.top.extend(c.top_logprobs if c.top_logprobs is not None else [None] * n)
        if self.entropy is not None:
            self.entropy.extend(c.entropy if c.entropy is not None else [None] * n)
        if self.routing is not None:
            r = c.routing_indices
            if r is None:
                self.routing.extend([None] * n)
            else:
                for i in range(min(len(r), prompt_len)):
                    self.routing[i] = r[i]
                extra = list(r[prompt_len:]) if len(r) > prompt_len else []
                self.routing.extend(extra)
                self.routing.extend([None] * (n - len(extra)))

    def truncate(self, n: int):
        for name in ("logprobs", "top", "entropy", "routing"):
            a = getattr(self, name)
            if a is not None:
                setattr(self, name, a[:n])


class UnifiedReactRunner:
    def __init__(self, backend: LLMBackend, mcp_executor: McpExecutor, config: LoopConfig,
                 encoding: HarmonyEncoding | None = None):
        self.backend = backend
        self.mcp_executor = mcp_executor
        self.config = config
        self.encoding = encoding or HarmonyEncoding()

    # ------------------------------------------------------------------ budget
    def _calculate_token_budget(self, context_len: int, generated: int) -> TokenBudget:
        c = self.config
        options = [(c.max_round_tokens, TruncationReason.ROUND_LIMIT),
                   (c.max_context_tokens - context_len, TruncationReason.CONTEXT_SPACE),
                   (c.max_total_tokens - generated, TruncationReason.GENERATION_QUOTA)]
        m, why = min(options, key=lambda x: x[0])
        return TokenBudget(max_tokens=max(0, m), limiting_factor=why)

    # ------------------------------------------------------------------ generation
    async def _generate(self, tokens: list[int], max_tokens: int, stop_event, record,
                        stop_ids: Optional[list[int]] = None) -> GenerationResult:
        stop_ids = stop_ids or self.encoding.stop_tokens_for_assistant_actions()
        if self.config.segment_temperature is not None and record is None:
            return await self._generate_segmented(tokens, max_tokens, stop_event, stop_ids)
        stream = self.config.use_streaming and not (record is not None and record.routing_indices)
        return await self.backend.generate(tokens, max_tokens, stop_ids, self.config.sampling,
                                           stream=stream, stop_event=stop_event, record=record)

    async def _generate_segmented(self, tokens, max_tokens, stop_event, stop_ids):
        """Header with header_temperature (stop at <|message|>), content with the channel /
        recipient temperature.  Segment metadata is attached to ``usage['segments']``."""
        seg_cfg = self.config.segment_temperature
        base = self.config.sampling
        out: list[int] = []
        segments = []
        header_s = base.model_copy(update={"temperature": seg_cfg.header_temperature})
        h = await self.backend.generate(tokens, max_tokens, stop_ids + [MESSAGE], header_s,
                                        stream=self.config.use_streaming, stop_event=stop_event)
        out += h.token_ids
        segments.append(SegmentMeta(phase="header", start=0, end=len(out),
                                    temperature=seg_cfg.header_temperature))
        if h.finish_reason in ("abort", "length") or not out or out[-1] != MESSAGE:
            h.usage = {"segments": [s.model_dump() for s in segments]}
            return h
        p = StreamableParser(self.encoding)
        for t in out:
            p.process(t)
        ch, rcp = p.header_fields()
        temp = seg_cfg.get_content_temperature(ch, rcp)
        c = await self.backend.generate(tokens + out, max_tokens - len(out), stop_ids,
                                        base.model_copy(update={"temperature": temp}),
                                        stream=self.config.use_streaming, stop_event=stop_event)
        segments.append(SegmentMeta(phase="content", start=len(out), end=len(out) + len(c.token_ids),
                                    temperature=temp, channel=ch, recipient=rcp))
        out += c.token_ids
        return GenerationResult(out, c.finish_reason, None, None, None, None,
                                {"segments": [s.model_dump() for s in segments]},
                                weight_version=c.weight_version or h.weight_version)

    # ------------------------------------------------------------------ steps
    @staticmethod
    def _assistant_step(start, end, ms, me, round_index, t0, completion, budget, weight_segments,
                        recipient=None, tool_input=None, parse_error=None) -> AssistantStep:
        segs = []
        usage = completion.usage if completion is not None else None
        if usage and "segments" in usage:
            segs = [SegmentMeta(**s) for s in usage["segments"]]
        return AssistantStep(start=start, end=end, message_start=ms, message_end=me,
                             round_index=round_index, created_at=t0, elapsed=time.time() - t0,
                             stop_reason=completion.finish_reason if completion else None,
                             truncation_reason=(budget.limiting_factor if completion is not None
                                                and completion.finish_reason == "length" else None),
                             recipient=recipient, tool_input=tool_input, usage=usage,
                             segments=segs, weight_segments=weight_segments, parse_error=parse_error)

    # ------------------------------------------------------------------ main loop
    async def run(self, conversation: Conversation, *, initial_tokens: Optional[list[int]] = None,
                  stop_event: Optional[asyncio.Event] = None, preserve_on_stop: bool = False,
                  record_config: Optional[RecordConfig] = None, rollout_id: Optional[str] = None,
                  force_final: bool = False) -> ReactResult:
        cfg = self.config
        enc = self.encoding
        messages: list[Message] = list(conversation.messages)
        tokens = list(initial_tokens) if initial_tokens is not None else \
            enc.render_conversation_for_completion(conversation, "assistant", cfg.auto_drop_analysis)
        force_tokens: list[int] = []
        if force_final:
            force_tokens = [CHANNEL] + enc.tok.encode("final")
            tokens += force_tokens
        acc = _Acc(len(tokens), record_config)
        steps: list = [InitStep(start=0, end=len(tokens), message_start=0, message_end=len(messages),
                                created_at=time.time())]
        round_index = 0
        tool_time = 0.0
        generated = 0
        errors: list[str] = []
        end_reason: Optional[EndReason] = None
        detail: Optional[str] = None
        parse_retries = 0
        round_ids: list[int] = []
        round_ws: list[WeightSegment] = []
        round_start: Optional[int] = None
        aborts: list[AbortRecord] = []
        n_aborts = 0
        while round_index < cfg.max_rounds and end_reason is None:
            if stop_event is not None and stop_event.is_set():
                end_reason, detail = EndReason.INTERRUPTED, "interrupted:external_stop"
                break
            budget = self._calculate_token_budget(len(tokens), generated)
            if not budget.can_generate:
                end_reason, detail = EndReason.TOKEN_LIMIT, _LIMIT_DETAIL[budget.limiting_factor]
                break
            t0 = time.time()
            try:
                c = await self._generate(tokens, budget.max_tokens, stop_event, record_config)
            except Exception as exc:  # noqa: BLE001
                logger.exception("LLM error: %s", exc)
                end_reason, detail = EndReason.ERROR, "error:llm_error"
                errors.append(str(exc))
                break
            if c.finish_reason == "abort" and not (stop_event is not None and stop_event.is_set()):
                # weight update in flight: keep the partial tokens and resume from them
                if round_start is None:
                    round_start = len(tokens)
                prompt_len = len(tokens)
                seg0 = len(round_ids)
                tokens += c.token_ids
                round_ids += c.token_ids
                acc.add_completion(c, prompt_len)
                if c.token_ids:
                    round_ws.append(WeightSegment(start=seg0, end=seg0 + len(c.token_ids),
                                                  weight_version=c.weight_version or "unknown"))
                aborts.append(AbortRecord(round_index=round_index, weight_version=c.weight_version,
                                          partial_token_count=len(c.token_ids), timestamp=time.time()))
                generated += len(c.token_ids)
                n_aborts += 1
                if n_aborts >= cfg.max_aborts:
                    end_reason, detail = EndReason.ERROR, f"error:max_aborts_exceeded:{n_aborts}"
                    errors.append(f"Abort count {n_aborts} exceeded max_aborts {cfg.max_aborts}")
                    break
                continue
            stopped = stop_event is not None and stop_event.is_set()
            if stopped and not preserve_on_stop:
                end_reason, detail = EndReason.INTERRUPTED, "interrupted:external_stop"
                break
            a_start = round_start if round_start is not None else len(tokens)
            seg0 = len(round_ids)
            prompt_len = len(tokens)
            tokens += c.token_ids
            generated += len(c.token_ids)
            round_ids += c.token_ids
            round_ws.append(WeightSegment(start=seg0, end=seg0 + len(c.token_ids),
                                          weight_version=c.weight_version or "unknown"))
            acc.add_completion(c, prompt_len)
            parse_ids = (force_tokens + round_ids) if (force_tokens and round_index == 0) else round_ids
            try:
                parsed = enc.parse_messages_from_completion_tokens(parse_ids, role="assistant")
                if not parsed:
                    raise ValueError("no message in completion")
            except Exception as exc:  # noqa: BLE001
                if not stopped and parse_retries < cfg.max_parse_retries:
                    tokens = tokens[:a_start]
                    acc.truncate(a_start)
                    generated -= len(round_ids)
                    round_ids, round_ws, round_start = [], [], None
                    parse_retries += 1
                    continue
                steps.append(self._assistant_step(a_start, len(tokens), len(messages), len(messages),
                                                  round_index, t0, c, budget, list(round_ws),
                                                  parse_error=str(exc)))
                if stopped:
                    end_reason, detail = EndReason.INTERRUPTED, "interrupted:external_stop"
                    errors.append(f"Parse failed during stop: {exc}")
                else:
                    end_reason, detail = EndReason.ERROR, "error:parse_error"
                    errors.append(str(exc))
                break
            ms = len(messages)
            messages.extend(parsed)
            me = len(messages)
            last = parsed[-1]
            if stopped:
                end_reason, detail = EndReason.INTERRUPTED, "interrupted:external_stop"
                break
            if c.finish_reason == "length":
                end_reason, detail = EndReason.TOKEN_LIMIT, _LIMIT_DETAIL[budget.limiting_factor]
                steps.append(self._assistant_step(a_start, len(tokens), ms, me, round_index, t0, c,
                                                  budget, list(round_ws), recipient=last.recipient))
                break
            text = (last.content or "").strip()
            recipient, channel = last.recipient, last.channel
            if recipient is None:
                if channel == "final":
                    end_reason, detail = EndReason.COMPLETED, "completed:final"
                else:
                    end_reason, detail = EndReason.ERROR, "error:no_final_channel"
                    errors.append(f"recipient=None but channel={channel}, expected channel=final")
                steps.append(self._assistant_step(a_start, len(tokens), ms, me, round_index, t0, c,
                                                  budget, list(round_ws)))
                break
            if not text:
                end_reason, detail = EndReason.ERROR, "error:invalid_tool_call"
                errors.append(f"recipient={recipient} but content is empty")
                steps.append(self._assistant_step(a_start, len(tokens), ms, me, round_index, t0, c,
                                                  budget, list(round_ws), recipient=recipient))
                break
            if channel == "final":
                end_reason, detail = EndReason.ERROR, "error:tool_call_in_final_channel"
                errors.append(f"recipient={recipient} but channel=final")
                steps.append(self._assistant_step(a_start, len(tokens), ms, me, round_index, t0, c,
                                                  budget, list(round_ws), recipient=recipient,
                                                  tool_input=text))
                break
            steps.append(self._assistant_step(a_start, len(tokens), ms, me, round_index, t0, c,
                                              budget, list(round_ws), recipient=recipient,
                                              tool_input=text))
            if stop_event is not None and stop_event.is_set():
                end_reason, detail = EndReason.INTERRUPTED, "interrupted:external_stop"
                break
            # ---------------- tool call
            t_tool = time.time()
            lim = cfg.max_total_tool_time
            if lim > 0 and tool_time >= lim:
                report = ToolCallReport(tool_name=recipient, tool_input=text,
                                        tool_output=(f"Error: tool time budget exceeded (used "
                                                     f"{tool_time:.1f}s / {lim:.1f}s limit)"),
                                        elapsed=0.0, error=ToolErrorType.TIMEOUT)
            else:
                report = await self.mcp_executor.call_tool(recipient, text)
                tool_time += report.elapsed
            tmsg = Message(role=recipient, content=report.tool_output, channel=channel,
                           recipient="assistant")
            tms = len(messages)
            messages.append(tmsg)
            ttoks = enc.render(tmsg) + [START] + enc.tok.encode("assistant")
            tstart = len(tokens)
            tokens += ttoks
            acc.pad(len(ttoks))
            steps.append(ToolStep(start=tstart, end=len(tokens), message_start=tms,
                                  message_end=len(messages), round_index=round_index,
                                  created_at=t_tool, elapsed=report.elapsed,
                                  tool_name=report.tool_name, tool_input=text,
                                  tool_output=report.tool_output, error=report.error,
                                  early_exit=report.early_exit,
                                  structured_output=report.structured_output))
            if report.early_exit:
                end_reason, detail = EndReason.TOOL_EARLY_EXIT, f"tool_early_exit:{report.tool_name}"
                break
            if report.error is not None and cfg.tool_error_strategy == "stop":
                end_reason, detail = EndReason.ERROR, f"error:tool_{report.error.value}"
                errors.append(f"Tool {report.tool_name} failed: {report.tool_output}")
                break
            round_ids, round_ws, round_start = [], [], None
            round_index += 1
        if end_reason is None:
            end_reason, detail = EndReason.MAX_ROUNDS, f"max_rounds:{cfg.max_rounds}"
        er = cfg.extra_round
        stopped = stop_event is not None and stop_event.is_set()
        if er is not None and not stopped and (
                (end_reason == EndReason.TOKEN_LIMIT and er.on_token_limit)
                or (end_reason == EndReason.MAX_ROUNDS and er.on_max_rounds)):
            ok = await self._extra_round(tokens, acc, messages, steps, round_index, record_config,
                                         stop_event, errors)
            if ok:
                detail = f"{detail}:extra_round"
        return ReactResult(end_reason=end_reason, end_reason_detail=detail, errors=errors,
                           tokens=tokens, logprobs=acc.logprobs, entropy=acc.entropy,
                           top_logprobs=acc.top, routing_indices=acc.routing, steps=steps,
                           conversation=Conversation(messages), total_tool_time=tool_time,
                           num_generated_tokens=generated, abort_records=aborts)

    async def _extra_round(self, tokens, acc, messages, steps, round_index, record, stop_event,
                           errors) -> bool:
        """Inject the budget notice as a user message and force a final-channel answer."""
        er = self.config.extra_round
        enc = self.encoding
        # close a dangling assistant header left by a tool step
        if tokens[-1:] and len(tokens) >= 2 and steps and isinstance(steps[-1], ToolStep):
            trim = 1 + len(enc.tok.encode("assistant"))
            del tokens[-trim:]
            acc.truncate(len(tokens))
        notice = Message(role="user", content=er.message)
        inject = enc.render(notice) + [START] + enc.tok.encode("assistant") + [CHANNEL] + \
            enc.tok.encode("final") + [MESSAGE]
        space = self.config.max_context_tokens - len(tokens) - len(inject)
        if space < er.min_budget:
            return False
        ms = len(messages)
        messages.append(notice)
        tokens += inject
        acc.pad(len(inject))
        t0 = time.time()
        try:
            c = await self._generate(tokens, min(er.budget, space), stop_event, record)
        except Exception as exc:  # noqa: BLE001
            errors.append(f"extra round failed: {exc}")
            return False
        a_start = prompt_len = len(tokens)  # the forced header is prompt, not generated

        tokens += c.token_ids
        acc.add_completion(c, prompt_len)
        text = enc.decode([t for t in c.token_ids if t < 199998])
        messages.append(Message(role="assistant", content=text.strip(), channel="final"))
        steps.append(self._assistant_step(a_start, len(tokens), ms, len(messages), round_index, t0, c,
                                          TokenBudget(er.budget, TruncationReason.ROUND_LIMIT),
                                          [WeightSegment(start=0, end=len(tokens) - a_start,
                                                         weight_version=c.weight_version or "unknown")]))
        return True
