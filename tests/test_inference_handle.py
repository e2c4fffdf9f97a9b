"""AgentHandle against a scripted sglang-compatible streaming server and the in-process Wordle
MCP server: tool rounds and events, pause/resume (stream closed and re-issued over the partial
tokens), stop, forced extra round with assistant prefill, message injection, probe, and
continue_from out of the dormant state."""
import asyncio
import json

from aiohttp import web
from aiohttp.test_utils import TestServer

from agent_factory_3_b200.envs import wordle
from agent_factory_3_b200.inference import AgentConfig, AgentHandle, EndReason, EventType, Phase
from agent_factory_3_b200.rollout.harmony import (CALL, CHANNEL, CONSTRAIN, END, MESSAGE, RETURN,
                                                  START, ByteTokenizer, HarmonyEncoding)

ENC = HarmonyEncoding(ByteTokenizer())
T = ENC.tok.encode


def tool_call(word):
    return ([CHANNEL] + T("analysis") + [MESSAGE] + T("think") + [END, START] + T("assistant")
            + [CHANNEL] + T("commentary to=wordle.guess ") + [CONSTRAIN] + T("json") + [MESSAGE]
            + T(json.dumps({"word": word})) + [CALL])


def final(text):
    return [CHANNEL] + T("final") + [MESSAGE] + T(text) + [RETURN]


class FakeServer:
    """Streams queued completions one token per chunk; a request whose prompt extends the
    previous prompt with a prefix of its completion continues that completion (re-issue)."""

    def __init__(self, outs, probe_outs=(), delay=0.002):
        self.outs, self.probe_outs, self.delay = list(outs), list(probe_outs), delay
        self.requests = []
        self.current = None

    async def generate(self, request):
        body = await request.json()
        prompt, sp = body["input_ids"], body["sampling_params"]
        self.requests.append(body)
        if not body.get("stream"):
            ids = self.probe_outs.pop(0)[:sp["max_new_tokens"]]
            return web.json_response({"output_ids": ids, "meta_info": {"finish_reason": {"type": "stop"}}})
        cont = None
        if self.current is not None:
            p0, script = self.current
            k = len(prompt) - len(p0)
            if k >= 0 and prompt[:len(p0)] == p0 and prompt[len(p0):] == script[:k]:
                cont = script[k:]
        if cont is None:
            script = self.outs.pop(0)
            self.current = (list(prompt), script)
            cont = script
        cont = cont[:sp["max_new_tokens"]]
        resp = web.StreamResponse(headers={"Content-Type": "text/event-stream"})
        await resp.prepare(request)
        try:
            for i, t in enumerate(cont):
                last = i == len(cont) - 1
                fr = ({"type": "stop"} if t in (RETURN, CALL) else {"type": "length"}) if last else None
                await resp.write(f"data: {json.dumps({'output_ids': [t], 'meta_info': {'finish_reason': fr}})}\n\n".encode())
                await asyncio.sleep(self.delay)
            await resp.write(b"data: [DONE]\n\n")
        except (ConnectionResetError, asyncio.CancelledError):
            pass
        return resp


async def _with_server(fake, fn):
    app = web.Application()
    app.router.add_post("/generate", fake.generate)
    srv = TestServer(app)
    await srv.start_server()
    try:
        return await fn(str(srv.make_url("")).rstrip("/"))
    finally:
        await srv.close()


def _handle(url, **kw):
    cfg = AgentConfig(server_url=url, max_rounds=kw.pop("max_rounds", 4), **kw)
    return AgentHandle(cfg, mcp_servers={"wordle": wordle.build_server("crane")}, encoding=ENC)


def test_tool_round_events_and_continue_from():
    fake = FakeServer([tool_call("slate"), final("the word is crane"), final("again")])

    async def run(url):
        h = _handle(url)
        await h.start("play wordle")
        kinds = [e.type async for e in h.events()]
        r = await h.join()
        assert r.end_reason == EndReason.COMPLETED and r.end_reason_detail == "completed:final"
        assert h.phase == Phase.DORMANT
        for k in (EventType.STARTED, EventType.ROUND_START, EventType.STREAM_CHUNK,
                  EventType.TOOL_CALL_START, EventType.TOOL_CALL_DONE, EventType.ROUND_DONE,
                  EventType.COMPLETED):
            assert k in kinds
        assert [s.type for s in r.steps] == ["init", "assistant", "tool", "assistant"]
        assert r.steps[2].tool_name == "guess" and "attempts" in r.steps[2].tool_output
        assert r.num_generated_tokens == len(tool_call("slate")) + len(final("the word is crane"))
        # the second request's prompt is the first completion plus the tool message
        assert fake.requests[1]["input_ids"][:len(fake.requests[0]["input_ids"])] == fake.requests[0]["input_ids"]
        await h.continue_from("once more")
        r2 = await h.join()
        assert r2.end_reason == EndReason.COMPLETED
        assert ENC.decode(fake.requests[2]["input_ids"]).count("once more") == 1
        await h.close()
        assert h.phase == Phase.COMPLETED

    asyncio.run(_with_server(fake, run))


def test_pause_resume_reissues_over_partial_tokens():
    long = final("x" * 80)
    fake = FakeServer([long], delay=0.003)

    async def run(url):
        h = _handle(url)
        await h.start("hi")
        seen = []
        async for e in h.events():
            seen.append(e.type)
            if e.type == EventType.STREAM_CHUNK and len(h.streaming_tokens) == 20:
                h.pause()
            if e.type == EventType.PAUSED:
                assert h.phase == Phase.PAUSED and len(h.streaming_tokens) >= 20
                h.resume()
        r = await h.join()
        assert EventType.PAUSED in seen and EventType.RESUMED in seen
        assert r.end_reason == EndReason.COMPLETED
        assert r.num_generated_tokens == len(long)
        assert len(fake.requests) == 2
        first, second = fake.requests[0]["input_ids"], fake.requests[1]["input_ids"]
        assert second[:len(first)] == first and len(second) - len(first) >= 20

    asyncio.run(_with_server(fake, run))


def test_stop_and_forced_extra_round_and_probe():
    fake = FakeServer([final("y" * 200), [MESSAGE] + T("42") + [RETURN], final("z" * 300)],
                      probe_outs=[[MESSAGE] + T("probe answer") + [RETURN]])

    async def run(url):
        h = _handle(url)
        await h.start("q")
        async for e in h.events():
            if e.type == EventType.STREAM_CHUNK and len(h.streaming_tokens) == 10:
                text = await h.probe("best guess?", budget=32)
                assert text == "probe answer" and h.phase == Phase.GENERATING
                h.force_extra_round(message="answer now")
        r = await h.join()
        assert r.end_reason == EndReason.COMPLETED and r.end_reason_detail == "completed:forced_final"
        extra_prompt = fake.requests[-1]["input_ids"]
        assert extra_prompt[-len(T("final")) - 1:] == [CHANNEL] + T("final")   # assistant prefill
        assert "answer now" in ENC.decode(extra_prompt)
        finals = [m for m in r.conversation.messages if m.channel == "final"]
        assert finals[-1].content == "42"
        probe_req = next(q for q in fake.requests if not q.get("stream"))
        assert "best guess?" in ENC.decode(probe_req["input_ids"])
        # stop during the continuation
        await h.continue_from("go on")
        async for e in h.events():
            if e.type == EventType.STREAM_CHUNK and len(h.streaming_tokens) == 5:
                h.stop()
        r2 = await h.join()
        assert r2.end_reason == EndReason.INTERRUPTED
        await h.close()

    asyncio.run(_with_server(fake, run))


def test_injection_and_max_rounds_extra_round():
    fake = FakeServer([tool_call("slate"), tool_call("trace"), [MESSAGE] + T("crane?") + [RETURN]])

    async def run(url):
        h = _handle(url, max_rounds=2)
        await h.start("play")
        injected = False
        async for e in h.events():
            if e.type == EventType.TOOL_CALL_DONE and not injected:
                h.inject_message("hint: it starts with c")
                injected = True
        r = await h.join()
        assert r.end_reason == EndReason.MAX_ROUNDS and r.end_reason_detail.endswith(":extra_round")
        # applied at the next round boundary after the call: after the first tool result, and
        # visible to every later request
        msgs = r.conversation.messages
        hint = next(i for i, m in enumerate(msgs) if m.content == "hint: it starts with c")
        first_tool = next(i for i, m in enumerate(msgs) if m.role == "wordle.guess")
        assert hint > first_tool and msgs[hint].role == "user"
        assert "hint: it starts with c" in ENC.decode(fake.requests[-1]["input_ids"])
        assert [m.content for m in r.conversation.messages if m.channel == "final"] == ["crane?"]
        await h.close()

    asyncio.run(_with_server(fake, run))
