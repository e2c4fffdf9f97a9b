"""CPU unit tests of the rollout-side pipeline: sample processor (trainability, baselines,
filters, routing gaps, weight versions), group-config factory (determinism, resume),
orchestrator batching with an in-process rollout function, engine-metrics parsing, rollout
saver/reader, checkpoint utilities and the HTML viewer."""
import asyncio
import time

import numpy as np
import pytest

from agent_factory_3_b200.orchestrator.orchestrator import Orchestrator
from agent_factory_3_b200.orchestrator.types import GroupResult, per_rollout
from agent_factory_3_b200.rollout.config import ConversationConfig, LoopConfig, RecordConfig
from agent_factory_3_b200.rollout.harmony import Conversation, Message
from agent_factory_3_b200.rollout.parallel.config import RolloutResult
from agent_factory_3_b200.rollout.types import (AssistantStep, EndReason, InitStep, ReactResult,
                                                WeightSegment)
from agent_factory_3_b200.trainer import checkpoint_utils as cu
from agent_factory_3_b200.trainer.engine_metrics import parse_loads_response, server_id_from_url
from agent_factory_3_b200.trainer.group_config_factory import GroupConfigFactory
from agent_factory_3_b200.trainer.rollout_saver import RolloutSaver
from agent_factory_3_b200.trainer.sample_processor import SampleProcessor
from agent_factory_3_b200.trainer.training_data_reader import iter_samples
from agent_factory_3_b200.visualizer import create_groups_viewer


def _result(rid, end=EndReason.COMPLETED, detail="completed:final", n_prompt=4, n_gen=3,
            versions=("1",), routing=True, gap=False):
    toks = list(range(n_prompt + n_gen))
    lp = [None] * n_prompt + [-0.5] * n_gen
    rt = [np.ones((2, 2), np.uint8)] * (n_prompt + n_gen) if routing else None
    if gap:
        rt = [np.ones((2, 2), np.uint8)] + [None] + [np.ones((2, 2), np.uint8)] * (n_prompt + n_gen - 2)
    segs, off = [], 0
    per = n_gen // len(versions)
    for i, v in enumerate(versions):
        e = n_gen if i == len(versions) - 1 else off + per
        segs.append(WeightSegment(start=off, end=e, weight_version=v))
        off = e
    rr = ReactResult(end_reason=end, end_reason_detail=detail, tokens=toks, logprobs=lp,
                     routing_indices=rt,
                     steps=[InitStep(start=0, end=n_prompt),
                            AssistantStep(start=n_prompt, end=n_prompt + n_gen, weight_segments=segs)],
                     conversation=Conversation([Message(role="user", content="hi")]),
                     total_tool_time=0.0, num_generated_tokens=n_gen)
    now = time.time()
    return RolloutResult(rollout_id=rid, result=rr, start_time=now - 1, end_time=now,
                         elapsed_time=1, server_url="http://x:1", success=True)


def test_sample_processor_rules():
    g1 = GroupResult("g1", [_result("a"), _result("b", versions=("2", "3")),
                            _result("c", EndReason.INTERRUPTED, "interrupted:external_stop")],
                     rewards=[1.0, 0.0, 1.0])
    g2 = GroupResult("g2", [_result("d"), _result("e")], rewards=[1.0, 1.0])          # all solved
    g3 = GroupResult("g3", [_result("f", EndReason.ERROR, "error:llm_error"),
                            _result("g", EndReason.ERROR, "error:parse_error"), _result("h")],
                     rewards=[0.0, 1.0, 0.0])
    samples, stats = SampleProcessor().process([g1, g2, g3])
    assert g1.trainable_mask == [True, True, False] and g1.reward_baseline == 0.5
    assert g1.advantages == [0.5, -0.5, 0.0]
    assert g2.filter_reason == "all_solved"
    assert g3.trainable_mask == [False, True, True]   # infra error out, parse error trainable
    assert g3.advantages == [0.0, 0.5, -0.5]
    ids = [s.sample_id for s in samples]
    assert ids == ["a", "b", "g", "h"]
    b = samples[1]
    assert b.oldest_weight_version == 2 and b.weight_version_token_counts == {2: 1, 3: 2}
    assert b.routing_indices.shape == (7, 2, 2)
    assert float(np.asarray(b.advantages)[-1]) == -0.5 and b.prompt_sequence_count == 2
    assert stats.filtered_all_solved == 1 and stats.total_samples == 4
    with pytest.raises(ValueError):
        SampleProcessor().to_sample(_result("x", gap=True).result, "x", "g", 1.0, 3, 1)


def test_group_factory_determinism_and_resume():
    ds = [{"prompt": f"p{i}", "mcp_config": None} for i in range(5)]
    kw = dict(dataset=ds, group_size=2, loop_config=LoopConfig(max_aborts=0),
              conv_config=ConversationConfig(), record_config=RecordConfig(), cache_salt_mode="per_group")
    f = GroupConfigFactory(**kw)
    it = iter(f)
    first = [next(it) for _ in range(7)]
    assert first[0].rollout_configs[0].loop_config.cache_salt == first[0].group_id
    seeds = {c.loop_config.sampling.seed for g in first for c in g.rollout_configs}
    assert len(seeds) == 14
    f2 = GroupConfigFactory(**kw)
    f2.load_state_dict(f.state_dict())
    # at-least-once: the group yielded last (possibly still in flight) is replayed on resume
    assert next(iter(f2)).group_id == first[-1].group_id


def test_orchestrator_batches_groups():
    async def fake_rollout(cfg, url):
        await asyncio.sleep(0.01)
        r = _result(cfg.rollout_id)
        r.server_url = url
        return r

    from agent_factory_3_b200.orchestrator.types import GroupConfig
    from agent_factory_3_b200.rollout.parallel.config import RolloutConfig
    groups = [GroupConfig(f"g{i}", [RolloutConfig(rollout_id=f"g{i}_r{j}", user_prompt="x",
                                                  loop_config=LoopConfig(max_aborts=0))
                                    for j in range(2)]) for i in range(5)]
    reward = per_rollout(lambda r, m: (float(r.rollout_id.endswith("0")), {"solved": 1.0}))
    orch = Orchestrator(["http://a:1", "http://b:2"], num_workers=2, worker_concurrency=2,
                        batch_size=4, reward_fn=reward, worker_mode="inproc", rollout_fn=fake_rollout,
                        poll_interval=0.05)

    async def run():
        out = []
        async for b in orch.run(groups):
            out.append(b)
        return out

    batches = asyncio.run(run())
    assert sum(len(b) for b in batches) == 5
    assert all(len(b) >= 2 for b in batches[:-1])
    g = batches[0][0]
    assert g.rewards in ([1.0, 0.0], [0.0, 1.0]) and g.results[0].reward_components == {"solved": 1.0}
    assert {r.server_url for b in batches for g in b for r in g.results} == {"http://a:1", "http://b:2"}


def test_metrics_saver_checkpoint_viewer(tmp_path):
    flat = parse_loads_response({"loads": [{"num_used_tokens": 5, "gen_throughput": 2.0,
                                            "memory": {"kv_cache_gb": 1.5}}]})
    assert flat["kv_used_tokens"] == 5 and flat["kv_cache_gb"] == 1.5
    assert np.isnan(flat["spec_accept_rate"]) and parse_loads_response({}) == {}
    assert server_id_from_url("http://10.0.0.1:30000") == "10.0.0.1_30000"
    g = GroupResult("g1", [_result("a"), _result("b")], rewards=[1.0, 0.0],
                    advantages=[0.5, -0.5], trainable_mask=[True, True])
    saver = RolloutSaver(tmp_path / "r")
    jp, hp, html = saver.save_batch([g], 0)
    assert jp.exists() and hp.exists() and "g1" in html and "<script>" in html
    p = saver.save_training_data([g], 0)
    recs = list(iter_samples(p))
    assert [r["rollout_id"] for r in recs] == ["a", "b"]
    assert recs[1]["advantages"][-1] == np.float16(-0.5)
    assert create_groups_viewer([g]).startswith("<!doctype html>")
    root = tmp_path / "ck"
    for step in (1, 2, 3):
        cu.write_meta(root / f"checkpoint_step_{step}", cu.CheckpointMeta(step=step, batch_idx=step))
    assert cu.find_latest_checkpoint(root).name == "checkpoint_step_3"
    cu.write_meta(root / "checkpoint_latest", cu.CheckpointMeta(step=9, batch_idx=9))
    assert cu.resolve_resume_path("latest", root).name == "checkpoint_latest"
    assert [p.name for p in cu.cleanup_old_checkpoints(root, 1)] == ["checkpoint_step_1", "checkpoint_step_2"]


def test_worker_lanes_bound_concurrency_and_report_failures(monkeypatch):
    """A worker with 3 lanes never runs more than 3 rollouts at once, turns a raising rollout
    into a failed result, answers every task exactly once and stops at the None marker
    without taking the tasks queued behind it."""
    import queue

    from agent_factory_3_b200.orchestrator import worker as W
    from agent_factory_3_b200.orchestrator.types import RolloutTask
    from agent_factory_3_b200.rollout.parallel.config import RolloutConfig

    state = {"active": 0, "peak": 0}

    async def fake_rollout(cfg, url):
        state["active"] += 1
        state["peak"] = max(state["peak"], state["active"])
        await asyncio.sleep(0.02)
        state["active"] -= 1
        if cfg.rollout_id == "t3":
            raise RuntimeError("boom")
        return _result(cfg.rollout_id)

    monkeypatch.setattr(W, "execute_rollout", fake_rollout)
    in_q, out_q = queue.Queue(), queue.Queue()
    for i in range(8):
        cfg = RolloutConfig(rollout_id=f"t{i}", user_prompt="p", loop_config=LoopConfig(),
                            conv_config=ConversationConfig(), record_config=RecordConfig())
        in_q.put(RolloutTask(config=cfg, server_url="http://x", group_id=f"g{i // 2}",
                             index_in_group=i % 2))
    in_q.put(None)
    in_q.put("left for another worker")
    asyncio.run(W._LaneWorker(in_q, out_q, 3, worker_id=0).run())
    got = [out_q.get_nowait() for _ in range(8)]
    assert out_q.empty() and state["peak"] == 3
    assert in_q.get_nowait() == "left for another worker"
    assert sorted((g, i) for g, i, _ in got) == sorted((f"g{i // 2}", i % 2) for i in range(8))
    failed = [r for _, _, r in got if not r.success]
    assert len(failed) == 1 and failed[0].rollout_id == "t3" and "boom" in failed[0].error


def test_server_pool_least_busy_and_release():
    import asyncio
    from agent_factory_3_b200.rollout.parallel.server_pool import ServerPool

    async def run():
        pool = ServerPool(["http://a", "http://b", "http://c"])
        got = [await pool.acquire() for _ in range(4)]
        assert got == ["http://a", "http://b", "http://c", "http://a"]   # ties go to list order
        await pool.release("http://b")
        await pool.release("http://b")          # never below zero
        assert await pool.acquire() == "http://b"
        assert pool.stats() == {"http://a": 2, "http://b": 1, "http://c": 1}
    asyncio.run(run())
    with pytest.raises(ValueError):
        ServerPool([])


def test_rollout_stats_and_monitor():
    from agent_factory_3_b200.rollout.parallel.execution_monitor import ExecutionMonitor
    from agent_factory_3_b200.rollout.parallel.postprocessing import (compute_stats_batch,
                                                                       validate_routing_indices)
    ok, bad = _result("a"), _result("b")
    bad.result.routing_indices[0] = np.full((2, 2), 200, np.uint8)   # expert id past 128
    out = compute_stats_batch([ok, bad], num_experts=128)
    assert out[0].routing_valid and not out[1].routing_valid
    assert out[0].completion_tokens_count == 3 and out[0].num_rounds == 1
    assert validate_routing_indices(ok.result, num_experts=2)
    assert not validate_routing_indices(ok.result, num_experts=1)
    mon = ExecutionMonitor(total=2, use_tqdm=False)
    for r in out:
        mon.update(r)
    s = mon.summary()
    assert s["done"] == 2 and s["generated_tokens"] == 6 and s["end_reasons"] == {"completed": 2}
    mon.close()
