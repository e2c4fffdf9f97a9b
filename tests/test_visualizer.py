"""Rollout viewer: page structure for live GroupResults (conversation by role and channel, tool
errors and early exits, failed rollouts with traceback, skip reasons, summary), HTML escaping,
and re-rendering a batch saved as JSON by RolloutSaver."""
import time

from agent_factory_3_b200.orchestrator.types import GroupResult
from agent_factory_3_b200.rollout.harmony import Conversation, Message
from agent_factory_3_b200.rollout.parallel.config import RolloutResult
from agent_factory_3_b200.rollout.types import (AssistantStep, EndReason, InitStep, ReactResult,
                                                ToolErrorType, ToolStep, WeightSegment)
from agent_factory_3_b200.trainer.rollout_saver import RolloutSaver
from agent_factory_3_b200.visualizer import create_groups_viewer, load_saved_batch


def _rollout(rid, end=EndReason.COMPLETED, detail="completed:final", tool_error=False):
    msgs = [Message(role="system", content="You are ChatGPT"),
            Message(role="developer", content="# Instructions\nplay <wordle>"),
            Message(role="user", content="Guess the word."),
            Message(role="assistant", content="thinking...", channel="analysis"),
            Message(role="assistant", content='{"word": "slate"}', channel="commentary",
                    recipient="wordle.guess"),
            Message(role="wordle.guess", content="S L A T E: _ _ A _ E"),
            Message(role="assistant", content="crane", channel="final")]
    steps = [InitStep(start=0, end=4),
             AssistantStep(start=4, end=8, weight_segments=[WeightSegment(start=0, end=4,
                                                                          weight_version="7")]),
             ToolStep(start=8, end=10, tool_name="wordle.guess", tool_input='{"word": "slate"}',
                      tool_output="S L A T E: _ _ A _ E",
                      error=ToolErrorType.TOOL_ERROR if tool_error else None, early_exit=True),
             AssistantStep(start=10, end=12)]
    rr = ReactResult(end_reason=end, end_reason_detail=detail, tokens=list(range(12)),
                     steps=steps, conversation=Conversation(msgs), total_tool_time=0.25,
                     num_generated_tokens=6)
    now = time.time()
    return RolloutResult(rollout_id=rid, result=rr, start_time=now - 2, end_time=now,
                         elapsed_time=2.0, server_url="http://e:1", success=True, num_rounds=2,
                         reward_components={"win": 1.0})


def _failed(rid):
    now = time.time()
    return RolloutResult(rollout_id=rid, result=None, start_time=now - 1, end_time=now,
                         elapsed_time=1.0, server_url="http://e:1", success=False,
                         error="ConnectionError: engine down", traceback="Traceback ...\nboom")


def _groups():
    g1 = GroupResult("e0_i0", [_rollout("r0"), _rollout("r1", tool_error=True)], rewards=[1.0, 0.0],
                     metadata={"target": "crane", "_private": 1})
    g1.advantages, g1.trainable_mask, g1.skip_reasons = [0.5, -0.5], [True, False], [None, "zero_loss"]
    g2 = GroupResult("e0_i1", [_failed("r2")], rewards=[0.0])
    return [g1, g2]


def test_viewer_page_structure():
    page = create_groups_viewer(_groups(), title="Batch <7>")
    assert page.startswith("<!doctype html>") and "Batch &lt;7&gt;" in page
    for i in ("d0_0", "d0_1", "d1_0"):
        assert f'<template id="{i}">' in page and f'data-d="{i}"' in page
    assert "assistant · commentary → wordle.guess" in page
    assert "tool · wordle.guess" in page and "early exit" in page
    assert "error: tool_error" in page
    assert "ConnectionError: engine down" in page and "traceback" in page
    assert "zero_loss" in page and "weight versions" in page and "win=1.000" in page
    assert "3 rollouts" in page and "2 groups" in page
    assert "play &lt;wordle&gt;" in page          # message bodies are escaped
    assert "_private" not in page
    assert 'id="filter"' in page and "keydown" in page


def test_viewer_renders_saved_batch(tmp_path):
    groups = _groups()
    saver = RolloutSaver(tmp_path, save_html=False)
    jp, _, _ = saver.save_batch(groups, 3)
    loaded = load_saved_batch(str(jp))
    assert [g.group_id for g in loaded] == ["e0_i0", "e0_i1"]
    page = create_groups_viewer(loaded, title="reloaded")
    for rid in ("r0", "r1", "r2"):
        assert f">{rid}<" in page
    assert "assistant · commentary → wordle.guess" in page

    from agent_factory_3_b200.visualizer.app import main
    main([str(jp), "-o", str(tmp_path / "out.html")])
    assert (tmp_path / "out.html").read_text().startswith("<!doctype html>")
