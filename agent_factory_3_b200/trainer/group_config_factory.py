"""Infinite, resumable stream of rollout groups from a dataset (reference:
trainer/group_config_factory.py:20-184).  Every epoch shuffles the dataset with seed
``base_seed + epoch``; a group holds ``group_size`` rollouts of one item, each with a seed
derived from its rollout id (md5) and an optional prefix-cache salt (per group or per
rollout).  ``state_dict`` / ``load_state_dict`` restore the position after a restart."""
from __future__ import annotations

import hashlib
import json
import random
from pathlib import Path
from typing import Any, Callable, Iterator, Literal

from ..orchestrator.types import GroupConfig
from ..rollout.config import ConversationConfig, LoopConfig, RecordConfig
from ..rollout.parallel.config import RolloutConfig


def load_dataset(path: str | Path) -> list[dict[str, Any]]:
    path = Path(path)
    if not path.exists():
        raise FileNotFoundError(f"Dataset file not found: {path}")
    if path.suffix == ".jsonl":
        data = [json.loads(ln) for ln in path.read_text().splitlines() if ln.strip()]
    elif path.suffix == ".json":
        data = json.loads(path.read_text())
        if not isinstance(data, list):
            raise ValueError(f"Expected a list in {path}")
    else:
        raise ValueError(f"Unsupported dataset format: {path.suffix} (expected .json or .jsonl)")
    if not data:
        raise ValueError(f"Empty dataset: {path}")
    return data


def deterministic_seed(rollout_id: str) -> int:
    return int(hashlib.md5(rollout_id.encode()).hexdigest()[:8], 16)


class GroupConfigFactory:
    def __init__(self, *, dataset, group_size: int, loop_config: LoopConfig,
                 conv_config: ConversationConfig, record_config: RecordConfig,
                 prompt_key: str = "prompt", mcp_config_key: str = "mcp_config",
                 base_seed: int = 42, prompt_fn: Callable[[dict, str], tuple[str, dict]] | None = None,
                 cache_salt_mode: Literal["none", "per_group", "per_rollout"] = "none",
                 server_affinity: bool = False):
        if isinstance(dataset, (str, Path)):
            dataset = load_dataset(dataset)
        if not dataset:
            raise ValueError("dataset cannot be empty")
        if group_size < 2:
            raise ValueError(f"group_size must be >= 2, got {group_size}")
        if cache_salt_mode not in ("none", "per_group", "per_rollout"):
            raise ValueError(f"bad cache_salt_mode {cache_salt_mode!r}")
        self.dataset = dataset
        self.group_size = group_size
        self.loop_config = loop_config
        self.conv_config = conv_config
        self.record_config = record_config
        self.prompt_key = prompt_key
        self.mcp_config_key = mcp_config_key
        self.base_seed = base_seed
        self.prompt_fn = prompt_fn
        self.cache_salt_mode = cache_salt_mode
        self.server_affinity = server_affinity
        self.current_epoch = 0
        self.current_position = 0

    def __iter__(self) -> Iterator[GroupConfig]:
        while True:
            rng = random.Random(self.base_seed + self.current_epoch)
            idx = list(range(len(self.dataset)))
            rng.shuffle(idx)
            for i in idx[self.current_position:]:
                yield self._make_group(f"e{self.current_epoch}_i{i}", self.dataset[i])
                self.current_position += 1
            self.current_epoch += 1
            self.current_position = 0

    def _make_group(self, gid: str, item: dict) -> GroupConfig:
        if self.prompt_fn is not None:
            prompt, extra = self.prompt_fn(item, gid)
            meta = {k: v for k, v in item.items() if not k.startswith("_")}
            meta.update(extra)
        else:
            prompt = item[self.prompt_key]
            meta = item
        mcp = item.get(self.mcp_config_key)
        overrides = item.get("_loop_overrides") or {}
        cfgs = []
        for j in range(self.group_size):
            rid = f"{gid}_r{j}"
            salt = gid if self.cache_salt_mode == "per_group" else (
                rid if self.cache_salt_mode == "per_rollout" else None)
            lc = self.loop_config.model_copy(update={
                "sampling": self.loop_config.sampling.model_copy(update={"seed": deterministic_seed(rid)}),
                "cache_salt": salt, **overrides})
            cfgs.append(RolloutConfig(rollout_id=rid, user_prompt=prompt, loop_config=lc,
                                      conv_config=self.conv_config, record_config=self.record_config,
                                      mcp_config=mcp, metadata=meta))
        return GroupConfig(group_id=gid, rollout_configs=cfgs, metadata=meta,
                           server_affinity=self.server_affinity)

    def state_dict(self) -> dict:
        return {"current_epoch": self.current_epoch, "current_position": self.current_position,
                "base_seed": self.base_seed, "dataset_size": len(self.dataset)}

    def load_state_dict(self, state: dict) -> None:
        if state.get("dataset_size", len(self.dataset)) != len(self.dataset):
            raise ValueError("dataset size changed since the checkpoint; cannot resume position")
        self.current_epoch = int(state["current_epoch"])
        self.current_position = int(state["current_position"])
