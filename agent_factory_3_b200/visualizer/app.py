"""Rollout viewer: a list of ``GroupResult`` -> one self-contained HTML page (inline CSS and JS,
no server, no external assets).  Reference: ``visualizer/app.py:127-304`` of the reference
(a two-pane rollout viewer with group cards, a rollout list and a conversation pane).

Layout:
* a header with the batch summary (groups, rollouts, task success rate, mean reward, trainable
  share, mean generated tokens, end-reason counts) and a filter box;
* a left pane with one card per group (id, mean reward, filter reason, metadata) listing its
  rollouts (status, reward, advantage, generated tokens, end reason; untrainable rollouts
  marked with their skip reason);
* a right pane showing the selected rollout: run facts (rounds, tokens, elapsed and tool time,
  weight versions, reward components, errors, aborts, traceback) and the conversation by role
  and channel -- system / developer configuration collapsed, assistant analysis / commentary /
  final with tool-call recipients, tool results with their errors and early exits, long bodies
  collapsible.
Each rollout's detail is rendered once into a hidden ``<template>``; clicking a rollout (or
``j`` / ``k``) shows it.  ``python -m agent_factory_3_b200.visualizer batch.json -o out.html``
renders a batch saved by ``RolloutSaver``.
"""
from __future__ import annotations

import html
import json
from typing import Any

from .assets import CSS, JS
from .views import GroupView, MessageView, RolloutView, Summary, group_views

LONG = 1200     # characters after which a body is collapsed behind a summary line


def _e(x: Any) -> str:
    return html.escape("" if x is None else str(x))


def _badge(text, kind: str = "") -> str:
    return f'<span class="badge {kind}">{_e(text)}</span>'


def _body(text: str, cls: str = "body") -> str:
    if len(text) <= LONG:
        return f'<div class="{cls}">{_e(text)}</div>'
    first = text[:160].replace("\n", " ")
    return (f'<details class="long"><summary>{_e(first)}… ({len(text)} chars)</summary>'
            f'<div class="{cls}">{_e(text)}</div></details>')


def _message(m: MessageView, tool_info: dict | None) -> str:
    if m.role in ("system", "developer"):
        return (f'<details class="msg {m.role}"><summary class="role">{_e(m.role)}</summary>'
                f'{_body(m.text)}</details>')
    cls, label, extra = m.role, m.role, ""
    if m.role == "assistant":
        ch = m.channel or "final"
        cls = f"assistant {ch}"
        label = f"assistant · {ch}"
        if m.recipient:
            label += f" → {m.recipient}"
            cls += " call"
    elif m.role == "tool":
        label = f"tool · {m.author or ''}"
        if tool_info:
            if tool_info.get("error"):
                cls += " error"
                extra += _badge(f"error: {tool_info['error']}", "bad")
            if tool_info.get("early_exit"):
                extra += _badge("early exit", "warn")
    return (f'<div class="msg {cls}"><div class="role">{_e(label)} {extra}</div>'
            f'{_body(m.text)}</div>')


def _facts(r: RolloutView) -> str:
    rows = [("rounds", r.num_rounds), ("generated tokens", r.gen_tokens),
            ("tokens", r.total_tokens), ("elapsed", f"{r.elapsed_s:.2f} s"),
            ("tool time", f"{r.tool_time_s:.2f} s"),
            ("end", f"{r.end_reason or 'failed'}" + (f" ({r.end_detail})" if r.end_detail else ""))]
    if r.weight_versions:
        rows.append(("weight versions", ", ".join(r.weight_versions)))
    if r.reward_components:
        rows.append(("reward components", ", ".join(f"{k}={v:.3f}" for k, v in
                                                    r.reward_components.items())))
    if r.skip_reason:
        rows.append(("not trained", r.skip_reason))
    out = "".join(f'<tr><th>{_e(k)}</th><td>{_e(v)}</td></tr>' for k, v in rows)
    extra = ""
    if r.error:
        extra += f'<div class="msg error"><div class="role">error</div>{_body(r.error)}</div>'
    for e in r.errors:
        extra += f'<div class="msg error"><div class="role">rollout error</div>{_body(e)}</div>'
    for a in r.aborts:
        extra += f'<div class="msg warn"><div class="role">abort</div>{_body(a)}</div>'
    if r.traceback:
        extra += (f'<details class="msg error"><summary class="role">traceback</summary>'
                  f'<pre>{_e(r.traceback)}</pre></details>')
    return f'<table class="facts">{out}</table>{extra}'


def _detail(r: RolloutView, idx: str) -> str:
    head = [f'<h2>{_e(r.rollout_id)}</h2>']
    if r.reward is not None:
        head.append(_badge(f"reward {r.reward:.3f}", "ok" if r.reward > 0 else ""))
    if r.advantage is not None:
        head.append(_badge(f"advantage {r.advantage:+.3f}"))
    head.append(_badge("success" if r.task_success else ("ran" if r.ok else "failed"),
                       "ok" if r.task_success else ("" if r.ok else "bad")))
    if r.trainable is not None:
        head.append(_badge("trainable" if r.trainable else "skipped",
                           "" if r.trainable else "warn"))
    # pair tool messages with their steps in order (one tool message per tool call)
    tools = iter(r.tools)
    msgs = []
    for m in r.messages:
        info = None
        if m.role == "tool":
            t = next(tools, None)
            info = None if t is None else {"error": t.error, "early_exit": t.early_exit}
        msgs.append(_message(m, info))
    return (f'<template id="d{idx}"><div class="detail">{"".join(head)}{_facts(r)}'
            f'<h3>conversation ({len(r.messages)} messages, {len(r.tools)} tool calls)</h3>'
            f'{"".join(msgs)}</div></template>')


def _row(r: RolloutView, idx: str) -> str:
    status = "ok" if r.task_success else ("fail" if r.ok else "bad")
    bits = [f'<span class="dot {status}"></span><span class="rid">{_e(r.rollout_id)}</span>']
    if r.reward is not None:
        bits.append(f'<span class="num">{r.reward:.2f}</span>')
    if r.advantage is not None:
        bits.append(f'<span class="num adv">{r.advantage:+.2f}</span>')
    bits.append(f'<span class="num">{r.gen_tokens} tok</span>')
    bits.append(f'<span class="end">{_e(r.end_reason or "failed")}</span>')
    skip = "" if r.trainable is None or r.trainable else " skipped"
    title = f' title="{_e(r.skip_reason)}"' if r.skip_reason else ""
    return f'<div class="row{skip}" data-d="d{idx}"{title}>{"".join(bits)}</div>'


def _card(g: GroupView, gi: int) -> str:
    badges = [_badge(f"mean reward {g.mean_reward:.3f}")]
    if g.filter_reason:
        badges.append(_badge(f"filtered: {g.filter_reason}", "warn"))
    meta = json.dumps(g.metadata, ensure_ascii=False)[:300] if g.metadata else ""
    rows = "".join(_row(r, f"{gi}_{ri}") for ri, r in enumerate(g.rollouts))
    return (f'<div class="group"><div class="gh"><b>{_e(g.group_id)}</b> {"".join(badges)}</div>'
            f'<div class="meta">{_e(meta)}</div>{rows}</div>')


def _summary(s: Summary) -> str:
    items = [f"{s.groups} groups", f"{s.rollouts} rollouts",
             f"success {100 * s.success_rate:.1f}%", f"mean reward {s.mean_reward:.3f}",
             f"mean generated {s.mean_gen_tokens:.0f} tok"]
    if s.trainable_fraction is not None:
        items.append(f"trainable {100 * s.trainable_fraction:.1f}%")
    ends = " ".join(_badge(f"{k} {v}") for k, v in s.end_reasons.items())
    return f'<div class="summary">{" · ".join(_e(i) for i in items)} <span>{ends}</span></div>'


def create_groups_viewer(group_results: list, title: str = "Rollouts") -> str:
    """Self-contained HTML of a batch of ``GroupResult`` (see the module docstring)."""
    groups, summary = group_views(group_results)
    cards = "".join(_card(g, gi) for gi, g in enumerate(groups))
    details = "".join(_detail(r, f"{gi}_{ri}") for gi, g in enumerate(groups)
                      for ri, r in enumerate(g.rollouts))
    return (f"<!doctype html><html><head><meta charset='utf-8'><title>{_e(title)}</title>"
            f"<style>{CSS}</style></head><body><header><h1>{_e(title)}</h1>{_summary(summary)}"
            f'<input id="filter" placeholder="filter groups and rollouts…"></header>'
            f'<main><nav id="list">{cards}</nav><section id="pane"><div class="empty">'
            f"Select a rollout (click, or j / k)</div></section></main>{details}"
            f"<script>{JS}</script></body></html>")


def load_saved_batch(path: str) -> list:
    """``GroupResult`` objects from a batch JSON written by ``RolloutSaver.save_batch``."""
    from ..orchestrator.types import GroupResult
    from ..rollout.parallel.config import RolloutResult
    rows = json.loads(open(path, encoding="utf-8").read())
    out = []
    for g in rows:
        results = [RolloutResult.model_validate(r) for r in g.get("results", [])]
        out.append(GroupResult(group_id=g["group_id"], results=results,
                               rewards=list(g.get("rewards", [])),
                               metadata=dict(g.get("metadata", {})),
                               advantages=list(g.get("advantages", [])),
                               trainable_mask=list(g.get("trainable_mask", [])),
                               filter_reason=g.get("filter_reason")))
    return out


def main(argv: list[str] | None = None) -> None:
    import argparse
    ap = argparse.ArgumentParser(description="render a saved rollout batch as HTML")
    ap.add_argument("batch_json")
    ap.add_argument("-o", "--output", default=None)
    ap.add_argument("--title", default=None)
    a = ap.parse_args(argv)
    groups = load_saved_batch(a.batch_json)
    out = a.output or a.batch_json.rsplit(".", 1)[0] + ".html"
    with open(out, "w", encoding="utf-8") as f:
        f.write(create_groups_viewer(groups, title=a.title or a.batch_json))
    print(out)
