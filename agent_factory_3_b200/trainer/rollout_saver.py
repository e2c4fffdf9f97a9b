"""Per-batch rollout dumps (reference: trainer/rollout_saver.py:24-365): JSON with full
conversations, a self-contained HTML viewer, and a compressed NPZ of the training data
(token ids int32, rollout log-probs float16 with NaN where not generated, completion mask,
advantages float16, routing uint8 with 255 for unknown, cu_seqlens, JSON metadata)."""
from __future__ import annotations

import json
import logging
from pathlib import Path

import numpy as np

from ..visualizer import create_groups_viewer

logger = logging.getLogger(__name__)
ROUTING_SENTINEL = 255


def _routing_array(react) -> np.ndarray | None:
    if react.routing_indices is None:
        return None
    first = next((x for x in react.routing_indices if x is not None), None)
    if first is None:
        return None
    f = np.asarray(first)
    arr = np.full((len(react.routing_indices), f.shape[0], f.shape[1]), ROUTING_SENTINEL, np.uint8)
    for i, x in enumerate(react.routing_indices):
        if x is not None:
            arr[i] = np.asarray(x, dtype=np.uint8)
    return arr


def _weight_version(react) -> str | None:
    vs = [ws.weight_version for s in react.steps if s.type.value == "assistant" for ws in s.weight_segments]
    return vs[0] if vs else None


class RolloutSaver:
    def __init__(self, output_dir: str | Path, save_routing_indices: bool = True,
                 save_html: bool = True):
        self.output_dir = Path(output_dir)
        self.output_dir.mkdir(parents=True, exist_ok=True)
        self.save_routing_indices = save_routing_indices
        self.save_html = save_html

    def save_batch(self, group_results: list, batch_index: int) -> tuple[Path, Path | None, str]:
        """JSON (+ HTML) of the batch; returns (json_path, html_path, html_string)."""
        rows = []
        for g in group_results:
            rows.append({
                "group_id": g.group_id, "rewards": g.rewards, "advantages": g.advantages,
                "trainable_mask": g.trainable_mask, "filter_reason": g.filter_reason,
                "metadata": {k: v for k, v in (g.metadata or {}).items()
                             if isinstance(v, (str, int, float, bool, list, dict))},
                "results": [json.loads(r.model_dump_json()) for r in g.results]})
        jp = self.output_dir / f"batch_{batch_index:04d}.json"
        jp.write_text(json.dumps(rows, ensure_ascii=False))
        html = create_groups_viewer(group_results, title=f"Batch {batch_index}")
        hp = None
        if self.save_html:
            hp = self.output_dir / f"batch_{batch_index:04d}.html"
            hp.write_text(html)
        return jp, hp, html

    def save_training_data(self, group_results: list, batch_index: int) -> Path | None:
        toks, lps, masks, advs, routes, meta = [], [], [], [], [], []
        offsets = [0]
        has_routing = False
        for g in group_results:
            for i, r in enumerate(g.results):
                react = r.result
                if react is None or react.logprobs is None or len(react.logprobs) != len(react.tokens):
                    continue
                T = len(react.tokens)
                mask = np.asarray(react.get_loss_mask(), np.uint8)
                adv = g.advantages[i] if i < len(g.advantages) else 0.0
                toks.append(np.asarray(react.tokens, np.int32))
                lps.append(np.array([np.nan if x is None else x for x in react.logprobs], np.float16))
                masks.append(mask)
                advs.append((mask * adv).astype(np.float16))
                if self.save_routing_indices:
                    rt = _routing_array(react)
                    has_routing |= rt is not None
                    routes.append(rt if rt is not None else T)
                offsets.append(offsets[-1] + T)
                meta.append({"rollout_id": r.rollout_id, "group_id": g.group_id,
                             "reward": g.rewards[i] if i < len(g.rewards) else 0.0,
                             "advantage": adv,
                             "trainable": g.trainable_mask[i] if i < len(g.trainable_mask) else False,
                             "weight_version": _weight_version(react),
                             "end_reason": react.end_reason.value, "filter_reason": g.filter_reason,
                             "seq_len": T,
                             "steps": [{"type": s.type.value, "start": s.start, "end": s.end}
                                       for s in react.steps]})
        if not toks:
            return None
        arrays = {"token_ids": np.concatenate(toks), "logprobs": np.concatenate(lps),
                  "completion_mask": np.concatenate(masks), "advantages": np.concatenate(advs),
                  "cu_seqlens": np.asarray(offsets, np.int32)}
        if has_routing:
            L, K = next(r.shape[1:] for r in routes if isinstance(r, np.ndarray))
            arrays["routing_indices"] = np.concatenate(
                [r if isinstance(r, np.ndarray) else np.full((r, L, K), ROUTING_SENTINEL, np.uint8)
                 for r in routes])
        arrays["metadata"] = np.frombuffer(json.dumps(meta, ensure_ascii=False).encode(), np.uint8).copy()
        p = self.output_dir / f"batch_{batch_index:04d}.npz"
        np.savez_compressed(p, **arrays)
        return p
