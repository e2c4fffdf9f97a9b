"""View model of the rollout viewer: what the page shows of each group and rollout, built from
the orchestrator's ``GroupResult`` objects (reference: ``visualizer/adapters/group_results.py``
and ``visualizer/core/types.py`` build the same information for their page).

Everything here is plain data (strings, numbers, lists), so the renderer never touches the
rollout objects and a batch saved as JSON by ``RolloutSaver`` renders the same way as a live one.
"""
from __future__ import annotations

import json
from collections import Counter
from dataclasses import dataclass, field
from typing import Any, Optional


@dataclass
class MessageView:
    role: str                      # system | developer | user | assistant | tool
    channel: Optional[str] = None  # analysis | commentary | final (assistant)
    recipient: Optional[str] = None
    author: Optional[str] = None   # tool name for tool messages
    text: str = ""


@dataclass
class ToolView:
    name: str
    input: str
    output: str
    error: Optional[str] = None
    early_exit: bool = False
    structured: Optional[dict] = None


@dataclass
class RolloutView:
    rollout_id: str
    ok: bool                       # the rollout ran without an infrastructure failure
    task_success: bool
    reward: Optional[float]
    advantage: Optional[float]
    trainable: Optional[bool]
    skip_reason: Optional[str]
    end_reason: Optional[str]
    end_detail: Optional[str]
    num_rounds: Optional[int]
    gen_tokens: int
    total_tokens: int
    elapsed_s: float
    tool_time_s: float
    weight_versions: list[str] = field(default_factory=list)
    reward_components: dict[str, float] = field(default_factory=dict)
    error: Optional[str] = None
    traceback: Optional[str] = None
    errors: list[str] = field(default_factory=list)
    aborts: list[str] = field(default_factory=list)
    messages: list[MessageView] = field(default_factory=list)
    tools: list[ToolView] = field(default_factory=list)


@dataclass
class GroupView:
    group_id: str
    rollouts: list[RolloutView]
    mean_reward: float
    filter_reason: Optional[str]
    metadata: dict[str, Any]


@dataclass
class Summary:
    groups: int
    rollouts: int
    success_rate: float
    mean_reward: float
    trainable_fraction: Optional[float]
    mean_gen_tokens: float
    end_reasons: dict[str, int]


def _get(obj, name, default=None):
    if isinstance(obj, dict):
        return obj.get(name, default)
    return getattr(obj, name, default)


def _text_of(content) -> str:
    if content is None:
        return ""
    if isinstance(content, str):
        return content
    if isinstance(content, (list, tuple)):
        return "\n".join(_text_of(c) for c in content)
    if isinstance(content, dict):
        if "text" in content:
            return str(content["text"])
        return json.dumps(content, ensure_ascii=False, indent=1)
    t = getattr(content, "text", None)
    return str(t) if t is not None else str(content)


def _enum_value(v):
    return getattr(v, "value", v)


def rollout_view(r, reward=None, advantage=None, trainable=None, skip_reason=None) -> RolloutView:
    res = _get(r, "result")
    versions: list[str] = []
    msgs: list[MessageView] = []
    tools: list[ToolView] = []
    aborts: list[str] = []
    if res is not None:
        conv = _get(res, "conversation")
        for m in (_get(conv, "messages", []) or []):
            role = str(_enum_value(_get(m, "role", "")))
            author = None
            if role not in ("system", "developer", "user", "assistant"):
                author, role = role, "tool"          # tool messages carry "<namespace.tool>"
            msgs.append(MessageView(role=role, channel=_get(m, "channel"),
                                    recipient=_get(m, "recipient"), author=author,
                                    text=_text_of(_get(m, "content"))))
        for s in (_get(res, "steps", []) or []):
            kind = str(_enum_value(_get(s, "type", "")))
            if kind == "tool":
                err = _get(s, "error")
                tools.append(ToolView(name=str(_get(s, "tool_name", "")),
                                      input=str(_get(s, "tool_input", "")),
                                      output=str(_get(s, "tool_output", "")),
                                      error=None if err is None else str(_enum_value(err)),
                                      early_exit=bool(_get(s, "early_exit", False)),
                                      structured=_get(s, "structured_output")))
            if kind == "assistant":
                for seg in (_get(s, "weight_segments", []) or []):
                    v = _get(seg, "weight_version")
                    if v is not None and str(v) not in versions:
                        versions.append(str(v))
        for a in (_get(res, "abort_records", []) or []):
            aborts.append(json.dumps(a if isinstance(a, dict) else
                                     (a.model_dump() if hasattr(a, "model_dump") else str(a)),
                                     default=str)[:300])
    return RolloutView(
        rollout_id=str(_get(r, "rollout_id", "?")), ok=bool(_get(r, "success", res is not None)),
        task_success=bool(res is not None and _get(res, "is_success", False)),
        reward=reward if reward is not None else _get(r, "weighted_reward"),
        advantage=advantage, trainable=trainable, skip_reason=skip_reason,
        end_reason=None if res is None else str(_enum_value(_get(res, "end_reason"))),
        end_detail=None if res is None else _get(res, "end_reason_detail"),
        num_rounds=_get(r, "num_rounds"),
        gen_tokens=int(_get(res, "num_generated_tokens", 0) or 0) if res is not None else 0,
        total_tokens=len(_get(res, "tokens", []) or []) if res is not None else 0,
        elapsed_s=float(_get(r, "elapsed_time", 0.0) or 0.0),
        tool_time_s=float(_get(res, "total_tool_time", 0.0) or 0.0) if res is not None else 0.0,
        weight_versions=versions, reward_components=dict(_get(r, "reward_components") or {}),
        error=_get(r, "error"), traceback=_get(r, "traceback"),
        errors=list(_get(res, "errors", []) or []) if res is not None else [],
        aborts=aborts, messages=msgs, tools=tools)


def group_views(group_results) -> tuple[list[GroupView], Summary]:
    """Views of every group and the page summary."""
    groups = []
    all_r: list[RolloutView] = []
    for g in group_results:
        results = list(_get(g, "results", []) or [])
        rewards = list(_get(g, "rewards", []) or [])
        advs = list(_get(g, "advantages", []) or [])
        mask = list(_get(g, "trainable_mask", []) or [])
        skips = list(_get(g, "skip_reasons", []) or [])
        views = []
        for i, r in enumerate(results):
            views.append(rollout_view(
                r, rewards[i] if i < len(rewards) else None,
                advs[i] if i < len(advs) else None,
                mask[i] if i < len(mask) else None,
                skips[i] if i < len(skips) else None))
        meta = {k: v for k, v in (_get(g, "metadata", {}) or {}).items()
                if isinstance(v, (str, int, float, bool)) and not str(k).startswith("_")}
        groups.append(GroupView(group_id=str(_get(g, "group_id", "?")), rollouts=views,
                                mean_reward=sum(rewards) / len(rewards) if rewards else 0.0,
                                filter_reason=_get(g, "filter_reason"), metadata=meta))
        all_r += views
    n = len(all_r)
    tr = [r.trainable for r in all_r if r.trainable is not None]
    rw = [r.reward for r in all_r if r.reward is not None]
    summary = Summary(
        groups=len(groups), rollouts=n,
        success_rate=sum(r.task_success for r in all_r) / n if n else 0.0,
        mean_reward=sum(rw) / len(rw) if rw else 0.0,
        trainable_fraction=sum(tr) / len(tr) if tr else None,
        mean_gen_tokens=sum(r.gen_tokens for r in all_r) / n if n else 0.0,
        end_reasons=dict(Counter(r.end_reason or "failed" for r in all_r).most_common()))
    return groups, summary
