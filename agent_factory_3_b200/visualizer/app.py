"""Rollout viewer: GroupResult list -> one self-contained HTML page (inline CSS and JS).

Each group is a card (id, rewards, advantages, filter reason); each rollout expands into its
conversation: system / developer / user prompts, assistant messages by channel (analysis,
commentary tool calls with recipient, final answers), tool outputs with errors and early
exits, plus end reason, token counts and abort records.  A filter box narrows the groups.
"""
from __future__ import annotations

import html
import json
from typing import Any

CSS = """
:root{--bg:#0f1117;--card:#171a23;--fg:#e6e6e6;--mute:#8a8f98;--acc:#6aa6ff;--ok:#3fb950;--bad:#f85149;--warn:#d29922}
body{background:var(--bg);color:var(--fg);font:14px/1.45 system-ui,-apple-system,Segoe UI,sans-serif;margin:0;padding:24px}
h1{font-size:20px;margin:0 0 12px}
.summary{color:var(--mute);margin-bottom:16px}
input#filter{background:var(--card);color:var(--fg);border:1px solid #333;border-radius:6px;padding:6px 10px;width:320px;margin-bottom:16px}
.group{background:var(--card);border-radius:10px;padding:12px 16px;margin-bottom:14px;border:1px solid #262a35}
.group h2{font-size:15px;margin:0 0 6px}
.badge{display:inline-block;border-radius:10px;padding:1px 8px;font-size:12px;margin-right:6px;background:#262a35}
.badge.ok{background:#12361f;color:var(--ok)}.badge.bad{background:#3d1618;color:var(--bad)}.badge.warn{background:#3a2c10;color:var(--warn)}
details.rollout{margin:6px 0;border-left:3px solid #333;padding-left:10px}
details.rollout>summary{cursor:pointer;color:var(--acc)}
.msg{margin:6px 0;padding:8px 10px;border-radius:6px;background:#1d212c;white-space:pre-wrap;word-break:break-word}
.msg .role{font-size:11px;color:var(--mute);text-transform:uppercase;letter-spacing:.05em;margin-bottom:3px}
.msg.system,.msg.developer{background:#1a1d26;color:#b8bcc6}
.msg.analysis{border-left:3px solid #555}.msg.commentary{border-left:3px solid var(--warn)}
.msg.final{border-left:3px solid var(--ok)}.msg.tool{border-left:3px solid var(--acc);background:#161b26}
.msg.error{border-left:3px solid var(--bad)}
.meta{color:var(--mute);font-size:12px}
"""

JS = """
document.getElementById('filter').addEventListener('input',e=>{const q=e.target.value.toLowerCase();
document.querySelectorAll('.group').forEach(g=>{g.style.display=g.innerText.toLowerCase().includes(q)?'':'none'})});
"""


def _e(x: Any) -> str:
    return html.escape(str(x))


def _badge(text, kind=""):
    return f'<span class="badge {kind}">{_e(text)}</span>'


def _render_rollout(r, reward, adv, trainable) -> str:
    res = getattr(r, "result", None)
    head = [f"<b>{_e(r.rollout_id)}</b>", _badge(f"reward {reward:.3f}", "ok" if reward > 0 else "")]
    if adv is not None:
        head.append(_badge(f"adv {adv:+.3f}"))
    if trainable is not None:
        head.append(_badge("trainable" if trainable else "skipped", "" if trainable else "warn"))
    if res is None:
        head.append(_badge("failed", "bad"))
        body = f'<div class="msg error">{_e(r.error or "no result")}</div>'
        return f'<details class="rollout"><summary>{" ".join(head)}</summary>{body}</details>'
    head.append(_badge(res.end_reason_detail, "ok" if res.is_success else "bad"))
    head.append(_badge(f"{res.num_generated_tokens} gen tok"))
    parts = []
    for m in res.conversation.messages:
        role = m.role
        cls = role if role in ("system", "developer", "user") else (
            "tool" if role not in ("assistant",) else (m.channel or "assistant"))
        label = role if role != "assistant" else f"assistant · {m.channel or ''}"
        if m.recipient and role == "assistant":
            label += f" → {m.recipient}"
        parts.append(f'<div class="msg {_e(cls)}"><div class="role">{_e(label)}</div>{_e(m.content)}</div>')
    tools = [s for s in res.steps if getattr(s, "type", None) == "tool" or s.type.value == "tool"]
    err = [s for s in tools if getattr(s, "error", None)]
    meta = (f'<div class="meta">tokens {len(res.tokens)} · tool time {res.total_tool_time:.2f}s · '
            f'tool errors {len(err)} · aborts {len(res.abort_records)} · errors {_e("; ".join(res.errors))}</div>')
    return (f'<details class="rollout"><summary>{" ".join(head)}</summary>{meta}'
            f'{"".join(parts)}</details>')


def create_groups_viewer(group_results: list, title: str = "Rollouts") -> str:
    cards = []
    n_roll = 0
    rewards_all = []
    for g in group_results:
        rewards = list(g.rewards)
        rewards_all += rewards
        advs = list(getattr(g, "advantages", []) or [None] * len(rewards))
        tm = list(getattr(g, "trainable_mask", []) or [None] * len(rewards))
        badges = [_badge(f"mean reward {sum(rewards) / max(1, len(rewards)):.3f}")]
        if getattr(g, "filter_reason", None):
            badges.append(_badge(f"filtered: {g.filter_reason}", "warn"))
        rolls = "".join(_render_rollout(r, w, a, t) for r, w, a, t in zip(g.results, rewards, advs, tm))
        n_roll += len(g.results)
        meta = _e(json.dumps({k: v for k, v in (g.metadata or {}).items()
                              if isinstance(v, (str, int, float, bool))})[:400])
        cards.append(f'<div class="group"><h2>{_e(g.group_id)}</h2>{"".join(badges)}'
                     f'<div class="meta">{meta}</div>{rolls}</div>')
    mean = sum(rewards_all) / max(1, len(rewards_all))
    return (f"<!doctype html><html><head><meta charset='utf-8'><title>{_e(title)}</title>"
            f"<style>{CSS}</style></head><body><h1>{_e(title)}</h1>"
            f'<div class="summary">{len(group_results)} groups · {n_roll} rollouts · mean reward {mean:.3f}</div>'
            f'<input id="filter" placeholder="filter groups…">{"".join(cards)}<script>{JS}</script></body></html>')
