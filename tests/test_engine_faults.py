"""Host-side fault injection in the engine server (CPU): dropped requests surface as HTTP 503
errors in the rollout backend, injected mid-generation aborts return the tokens produced so far
with finish reason "abort" (streaming and not), latency is added, and the engine frees the
aborted requests' pages."""
import asyncio
import time

import aiohttp
import pytest
from aiohttp.test_utils import TestClient, TestServer

from agent_factory_3_b200.engine.faults import FaultPlan
from agent_factory_3_b200.engine.scheduler import Engine
from agent_factory_3_b200.engine.server import build_app
from agent_factory_3_b200.rollout.config import SamplingParams
from agent_factory_3_b200.rollout.llm_backend.sglang_backend import SGLangBackend
from tests.test_engine import tiny_model


def test_fault_plan_parse():
    p = FaultPlan.parse("drop=0.25, delay_ms=5,abort_after=3,abort_rate=1,seed=7")
    assert (p.drop, p.delay_ms, p.abort_after, p.abort_rate, p.seed) == (0.25, 5.0, 3, 1.0, 7)
    with pytest.raises(ValueError):
        FaultPlan.parse("explode=1")
    hits = sum(FaultPlan(drop=0.5, seed=3).should_drop() for _ in range(1))
    assert hits in (0, 1)


def _run(plan, coro_fn):
    eng = Engine(tiny_model(), num_pages=64, page_size=8).start()

    async def main():
        client = TestClient(TestServer(build_app(eng, faults=plan)))
        await client.start_server()
        try:
            url = str(client.make_url("")).rstrip("/")
            backend = SGLangBackend(url)
            try:
                return await coro_fn(backend)
            finally:
                await backend.close()
        finally:
            await client.close()

    try:
        return asyncio.run(main()), eng
    finally:
        eng.stop()


def test_dropped_request_is_an_http_error():
    async def go(b):
        with pytest.raises(aiohttp.ClientResponseError) as e:
            await b.generate(list(range(3, 12)), 5, [], SamplingParams(temperature=0.0))
        return e.value.status
    status, _ = _run(FaultPlan(drop=1.0), go)
    assert status == 503


@pytest.mark.parametrize("stream", [False, True])
def test_injected_abort_returns_partial_tokens(stream):
    plan = FaultPlan(abort_after=3, abort_rate=1.0, delay_ms=20)

    async def go(b):
        t0 = time.perf_counter()
        r = await b.generate(list(range(3, 12)), 10, [], SamplingParams(temperature=0.0),
                             stream=stream)
        return r, time.perf_counter() - t0
    (res, dt), eng = _run(plan, go)
    assert res.finish_reason == "abort"
    assert len(res.token_ids) == 3
    assert dt >= 0.02
    assert plan.aborted == 1
    assert eng.kv.usage() == 0.0 or not eng.running
