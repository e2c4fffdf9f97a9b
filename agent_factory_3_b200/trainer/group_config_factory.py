"""Endless, resumable stream of rollout groups drawn from a dataset.

Contract (kept equal to the reference's trainer/group_config_factory.py:20-184 so runs line
up): the constructor keywords; every epoch visits the dataset in the order of
``random.Random(base_seed + epoch).shuffle``; group ids are ``e{epoch}_i{index}`` and rollout
ids ``{group}_r{j}``; each rollout's sampling seed is the first 32 bits of the md5 of its id;
dataset items may carry ``_loop_overrides`` (LoopConfig fields for that item) and
``_``-prefixed private keys that a ``prompt_fn`` hides from the metadata; the optional
prefix-cache salt is the group id or the rollout id.  ``state_dict`` records the position of
the group handed out LAST, so a resumed run replays it (at-least-once: that group may still
have been in flight when the checkpoint was written).

Design: ``_EpochOrder`` owns the seeded permutation and the cursor; ``_build_rollout`` turns
(group, item, j) into one RolloutConfig; the factory only wires the two together.
"""
from __future__ import annotations

import hashlib
import json
import random
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Callable, Iterator, Literal

from ..orchestrator.types import GroupConfig
from ..rollout.config import ConversationConfig, LoopConfig, RecordConfig
from ..rollout.parallel.config import RolloutConfig

SaltMode = Literal["none", "per_group", "per_rollout"]


def load_dataset(path: str | Path) -> list[dict[str, Any]]:
    """Items of a ``.json`` (one list) or ``.jsonl`` (one object per line) file."""
    path = Path(path)
    if not path.is_file():
        raise FileNotFoundError(f"no dataset at {path}")
    text = path.read_text()
    if path.suffix == ".jsonl":
        items = [json.loads(line) for line in text.splitlines() if line.strip()]
    elif path.suffix == ".json":
        items = json.loads(text)
        if not isinstance(items, list):
            raise ValueError(f"{path}: the top level must be a JSON list of items")
    else:
        raise ValueError(f"{path}: dataset files must end in .json or .jsonl")
    if not items:
        raise ValueError(f"{path} holds no items")
    return items


def deterministic_seed(rollout_id: str) -> int:
    """Sampling seed of a rollout: the first 8 hex digits of md5(rollout_id)."""
    return int(hashlib.md5(rollout_id.encode()).hexdigest()[:8], 16)


@dataclass
class _EpochOrder:
    """Seeded visiting order of ``n`` items, one permutation per epoch, with a cursor."""
    n: int
    base_seed: int
    epoch: int = 0
    cursor: int = 0

    def permutation(self) -> list[int]:
        order = list(range(self.n))
        random.Random(self.base_seed + self.epoch).shuffle(order)
        return order

    def walk(self) -> Iterator[tuple[int, int]]:
        """(epoch, item index) forever; the cursor counts items already handed out."""
        while True:
            order = self.permutation()
            while self.cursor < self.n:
                yield self.epoch, order[self.cursor]
                self.cursor += 1
            self.epoch, self.cursor = self.epoch + 1, 0


def _salt(mode: SaltMode, group_id: str, rollout_id: str) -> str | None:
    return {"none": None, "per_group": group_id, "per_rollout": rollout_id}[mode]


class GroupConfigFactory:
    """Iterating yields GroupConfig objects without end (see the module docstring)."""

    def __init__(self, *, dataset, group_size: int, loop_config: LoopConfig,
                 conv_config: ConversationConfig, record_config: RecordConfig,
                 prompt_key: str = "prompt", mcp_config_key: str = "mcp_config",
                 base_seed: int = 42, prompt_fn: Callable[[dict, str], tuple[str, dict]] | None = None,
                 cache_salt_mode: SaltMode = "none", server_affinity: bool = False):
        items = load_dataset(dataset) if isinstance(dataset, (str, Path)) else list(dataset or [])
        if not items:
            raise ValueError("the dataset has no items")
        if group_size < 2:
            raise ValueError(f"a group needs at least 2 rollouts to compare (group_size={group_size})")
        if cache_salt_mode not in ("none", "per_group", "per_rollout"):
            raise ValueError(f"cache_salt_mode must be none / per_group / per_rollout, "
                             f"not {cache_salt_mode!r}")
        self.dataset = items
        self.group_size = group_size
        self.loop_config, self.conv_config, self.record_config = loop_config, conv_config, record_config
        self.prompt_key, self.mcp_config_key = prompt_key, mcp_config_key
        self.prompt_fn = prompt_fn
        self.cache_salt_mode: SaltMode = cache_salt_mode
        self.server_affinity = server_affinity
        self._order = _EpochOrder(len(items), base_seed)

    # the position, as the reference names it (read by checkpoints and logs)
    @property
    def base_seed(self) -> int:
        return self._order.base_seed

    @property
    def current_epoch(self) -> int:
        return self._order.epoch

    @property
    def current_position(self) -> int:
        return self._order.cursor

    def __iter__(self) -> Iterator[GroupConfig]:
        for epoch, idx in self._order.walk():
            yield self.group(f"e{epoch}_i{idx}", self.dataset[idx])

    # -- one group -------------------------------------------------------------------
    def _prompt_and_meta(self, item: dict, group_id: str) -> tuple[str, dict]:
        if self.prompt_fn is None:
            return item[self.prompt_key], item
        prompt, extra = self.prompt_fn(item, group_id)
        public = {k: v for k, v in item.items() if not k.startswith("_")}
        return prompt, {**public, **extra}

    def _build_rollout(self, group_id: str, j: int, prompt: str, meta: dict, item: dict) -> RolloutConfig:
        rid = f"{group_id}_r{j}"
        sampling = self.loop_config.sampling.model_copy(update={"seed": deterministic_seed(rid)})
        update = {"sampling": sampling, "cache_salt": _salt(self.cache_salt_mode, group_id, rid)}
        update.update(item.get("_loop_overrides") or {})
        return RolloutConfig(rollout_id=rid, user_prompt=prompt,
                             loop_config=self.loop_config.model_copy(update=update),
                             conv_config=self.conv_config, record_config=self.record_config,
                             mcp_config=item.get(self.mcp_config_key), metadata=meta)

    def group(self, group_id: str, item: dict) -> GroupConfig:
        """The GroupConfig of one dataset item under the id ``group_id``."""
        prompt, meta = self._prompt_and_meta(item, group_id)
        rollouts = [self._build_rollout(group_id, j, prompt, meta, item)
                    for j in range(self.group_size)]
        return GroupConfig(group_id=group_id, rollout_configs=rollouts, metadata=meta,
                           server_affinity=self.server_affinity)

    # -- checkpointing ---------------------------------------------------------------
    def state_dict(self) -> dict:
        return {"current_epoch": self._order.epoch, "current_position": self._order.cursor,
                "base_seed": self._order.base_seed, "dataset_size": len(self.dataset)}

    def load_state_dict(self, state: dict) -> None:
        size = state.get("dataset_size", len(self.dataset))
        if size != len(self.dataset):
            raise ValueError(f"checkpoint was taken over {size} items, the dataset now has "
                             f"{len(self.dataset)}; the position cannot be restored")
        self._order.epoch = int(state["current_epoch"])
        self._order.cursor = int(state["current_position"])
