"""ReAct runner over harmony tokens with a scripted LLM backend and the in-process Wordle MCP
server: tool calls, early exit, abort/resume weight segments, routing accumulation, extra
round, serialisation round trip."""
import asyncio
import json

import numpy as np

from agent_factory_3_b200.envs import wordle
from agent_factory_3_b200.rollout.config import (ConversationConfig, ExtraRoundConfig, LoopConfig,
                                                 RecordConfig)
from agent_factory_3_b200.rollout.conversation_builder import ConversationBuilder
from agent_factory_3_b200.rollout.harmony import (CALL, CHANNEL, CONSTRAIN, END, MESSAGE, RETURN,
                                                  START, ByteTokenizer, HarmonyEncoding, Message)
from agent_factory_3_b200.rollout.llm_backend.types import GenerationResult
from agent_factory_3_b200.rollout.mcp_client import McpClient
from agent_factory_3_b200.rollout.mcp_executor import McpExecutor
from agent_factory_3_b200.rollout.parallel.config import RolloutConfig
from agent_factory_3_b200.rollout.parallel.executor import execute_rollout
from agent_factory_3_b200.rollout.runner import UnifiedReactRunner
from agent_factory_3_b200.rollout.types import EndReason, ReactResult, StepType

ENC = HarmonyEncoding(ByteTokenizer())
T = ENC.tok.encode


def tool_call(word):
    return ([CHANNEL] + T("analysis") + [MESSAGE] + T("think") + [END, START] + T("assistant")
            + [CHANNEL] + T("commentary to=wordle.guess ") + [CONSTRAIN] + T("json") + [MESSAGE]
            + T(json.dumps({"word": word})) + [CALL])


def final(text):
    return [CHANNEL] + T("final") + [MESSAGE] + T(text) + [RETURN]


class Scripted:
    """Returns queued completions; records the prompts it saw."""

    def __init__(self, outs, L=2, K=2):
        self.outs = list(outs)
        self.prompts = []
        self.L, self.K = L, K

    async def generate(self, prompt, max_tokens, stop, sampling, *, stream=False, stop_event=None,
                       record=None):
        self.prompts.append(list(prompt))
        o = self.outs.pop(0)
        ids, fr, ver = o if isinstance(o, tuple) else (o, "stop", "v0")
        ids = ids[:max_tokens]
        lp = [-0.5] * len(ids) if record and record.logprobs else None
        rt = None
        if record and record.routing_indices:
            n = len(prompt) + len(ids) - 1
            rt = np.full((n, self.L, self.K), 3, np.uint8)
        return GenerationResult(ids, fr, lp, None, rt, 0, None, None, ver)

    async def close(self):
        pass


async def _run(outs, loop_kw=None, record=None, target="crane"):
    server = wordle.build_server(target)
    async with McpClient(server) as client:
        ex = McpExecutor({"wordle": client})
        tc = await ex.get_tool_configs()
        conv = ConversationBuilder(ConversationConfig(dev_instructions="Play wordle.")).build(
            "Guess the word.", tc)
        be = Scripted(outs)
        cfg = LoopConfig(max_aborts=5, **(loop_kw or {}))
        res = await UnifiedReactRunner(be, ex, cfg, ENC).run(conv, record_config=record)
        return res, be, server


def test_tool_calls_and_early_exit():
    res, be, server = asyncio.run(_run([tool_call("slate"), tool_call("crane")]))
    assert res.end_reason == EndReason.TOOL_EARLY_EXIT
    tools = res.get_tool_steps()
    assert len(tools) == 2 and tools[-1].structured_output["won"] is True
    assert len(res.get_assistant_steps()) == 2
    # the developer message renders the tool namespace
    dev = ENC.decode(res.tokens[:res.steps[0].end])
    assert "namespace wordle" in dev and "type guess" in dev
    # loss mask covers exactly the generated tokens
    mask = res.get_loss_mask()
    assert sum(mask) == res.num_generated_tokens
    # the second prompt is the first prompt + completion + tool message + <|start|>assistant
    assert be.prompts[1][: len(be.prompts[0])] == be.prompts[0]


def test_final_answer_and_serialisation():
    res, _, _ = asyncio.run(_run([final("The word is crane.")],
                                 record=RecordConfig(logprobs=True, routing_indices=True)))
    assert res.end_reason == EndReason.COMPLETED
    assert res.conversation.messages[-1].channel == "final"
    assert res.routing_indices is not None and len(res.routing_indices) == len(res.tokens)
    back = ReactResult.model_validate(json.loads(res.model_dump_json()))
    assert back.tokens == res.tokens
    assert back.end_reason == res.end_reason
    n = sum(1 for r in res.routing_indices if r is not None)
    assert sum(1 for r in back.routing_indices if r is not None) == n
    assert back.logprobs[-1] == res.logprobs[-1]


def test_abort_resume_weight_segments():
    full = final("answer")
    outs = [(full[:3], "abort", "v0"), (full[3:], "stop", "v1")]
    res, be, _ = asyncio.run(_run(outs, record=RecordConfig(logprobs=True)))
    assert res.end_reason == EndReason.COMPLETED
    step = res.get_assistant_steps()[0]
    assert [w.weight_version for w in step.weight_segments] == ["v0", "v1"]
    assert step.weight_segments[0].end == 3 and step.weight_segments[1].start == 3
    assert len(res.abort_records) == 1
    # the resumed request continues from the partial tokens
    assert be.prompts[1] == be.prompts[0] + full[:3]


def test_errors_and_extra_round():
    # tool call in the final channel is an error
    bad = [CHANNEL] + T("final to=wordle.guess") + [MESSAGE] + T('{"word":"crane"}') + [CALL]
    res, _, _ = asyncio.run(_run([bad]))
    assert res.end_reason == EndReason.ERROR and res.end_reason_detail == "error:tool_call_in_final_channel"
    # max rounds then a forced final answer
    res, be, _ = asyncio.run(_run([tool_call("slate"), T("It is crane.") + [RETURN]],
                                  loop_kw={"max_rounds": 1, "extra_round": ExtraRoundConfig(budget=64, min_budget=8)}))
    assert res.end_reason == EndReason.MAX_ROUNDS
    assert res.end_reason_detail.endswith(":extra_round")
    assert res.conversation.messages[-1].content == "It is crane."
    assert any(m.role == "user" and "budget" in m.content for m in res.conversation.messages)


def test_execute_rollout_with_stdio_server(tmp_path):
    import sys
    cfg = RolloutConfig(rollout_id="r0", user_prompt="Guess.",
                        mcp_config={"mcpServers": {"wordle": {
                            "command": sys.executable,
                            "args": ["-m", "agent_factory_3_b200.envs.wordle", "--target", "crane"]}}},
                        loop_config=LoopConfig(max_aborts=0))
    r = asyncio.run(execute_rollout(cfg, "http://unused", backend=Scripted([tool_call("crane")]),
                                    encoding=ENC))
    assert r.success, r.error
    assert r.result.end_reason == EndReason.TOOL_EARLY_EXIT


def test_harmony_roundtrip():
    msgs = [Message(role="assistant", content="hi", channel="analysis"),
            Message(role="assistant", content='{"a":1}', channel="commentary",
                    recipient="functions.f", content_type="json", end=CALL)]
    ids = []
    for m in msgs:
        ids += ENC.render(m)
    # completion tokens start after "<|start|>assistant"
    comp = ids[1 + len(T("assistant")):]
    out = ENC.parse_messages_from_completion_tokens(comp)
    assert [(m.channel, m.recipient, m.content, m.content_type) for m in out] == \
        [("analysis", None, "hi", None), ("commentary", "functions.f", '{"a":1}', "json")]


def test_rollout_package_exports_the_reference_names():
    import agent_factory_3_b200.rollout as R
    names = {"ConversationConfig", "ExtraRoundConfig", "LoopConfig", "RecordConfig", "SamplingParams",
             "SegmentTemperatureConfig", "EndReason", "StepType", "TruncationReason", "TokenBudget",
             "SegmentMeta", "BaseStep", "InitStep", "AssistantStep", "ToolStep", "Step",
             "ReactResult", "McpExecutor", "ToolCallReport", "ToolErrorType", "ConversationBuilder",
             "UnifiedReactRunner", "CompletionResult", "RolloutConfig", "RolloutResult",
             "execute_rollout"}
    assert names <= set(R.__all__)
    assert all(getattr(R, n) is not None for n in names)
    from agent_factory_3_b200.rollout.runner import UnifiedReactRunner
    assert R.UnifiedReactRunner is UnifiedReactRunner


def test_vllm_backend_against_a_fake_openai_server():
    """Token ids in, token ids and log-probs out through /v1/completions (the client that the
    reference keeps for OpenAI-style servers)."""
    from aiohttp import web
    from aiohttp.test_utils import TestServer

    from agent_factory_3_b200.rollout.config import RecordConfig, SamplingParams
    from agent_factory_3_b200.rollout.llm_backend.vllm_backend import VLLMBackend
    seen = {}

    async def completions(request):
        body = await request.json()
        seen.update(body)
        return web.json_response({
            "choices": [{"finish_reason": "stop",
                         "logprobs": {"tokens": ["token_id:7", "token_id:9"],
                                      "token_logprobs": [-0.25, -1.5]}}],
            "usage": {"prompt_tokens": 3, "completion_tokens": 2}})

    async def run():
        app = web.Application()
        app.router.add_post("/v1/completions", completions)
        srv = TestServer(app)
        await srv.start_server()
        try:
            be = VLLMBackend(str(srv.make_url("")), "gpt-oss")
            r = await be.generate([1, 2, 3], 16, [200002], SamplingParams(temperature=0.5, top_k=20,
                                                                          seed=4),
                                  record=RecordConfig(logprobs=True))
            await be.close()
            return r
        finally:
            await srv.close()
    r = asyncio.run(run())
    assert r.token_ids == [7, 9] and r.logprobs == [-0.25, -1.5] and r.finish_reason == "stop"
    assert seen["prompt"] == [1, 2, 3] and seen["top_k"] == 20 and seen["seed"] == 4
    assert seen["stop_token_ids"] == [200002] and seen["logprobs"] == 1
