"""Run checkpoints: ``checkpoint_latest`` / ``checkpoint_step_N`` directories holding the
adapter (or trainable params), ``training_state.pt`` and an atomically written
``checkpoint_meta.json`` (step, batch index, dataset-factory position, wandb run id)
(reference: trainer/checkpoint_utils.py:17-99)."""
from __future__ import annotations

import json
import os
import re
import shutil
from pathlib import Path
from typing import Any, Optional

from pydantic import BaseModel

META = "checkpoint_meta.json"
LATEST = "checkpoint_latest"


class CheckpointMeta(BaseModel):
    step: int
    batch_idx: int
    factory_state: Optional[dict[str, Any]] = None
    wandb_run_id: Optional[str] = None
    weight_version: Optional[str] = None


def write_meta(ckpt_dir: str | Path, meta: CheckpointMeta) -> None:
    d = Path(ckpt_dir)
    d.mkdir(parents=True, exist_ok=True)
    tmp = d / (META + ".tmp")
    tmp.write_text(meta.model_dump_json(indent=2))
    os.replace(tmp, d / META)


def read_meta(ckpt_dir: str | Path) -> Optional[CheckpointMeta]:
    p = Path(ckpt_dir) / META
    if not p.exists():
        return None
    return CheckpointMeta.model_validate_json(p.read_text())


def find_latest_checkpoint(checkpoint_root: str | Path) -> Optional[Path]:
    root = Path(checkpoint_root)
    if (root / LATEST / META).exists():
        return root / LATEST
    steps = list_periodic(root)
    return steps[-1] if steps else None


def list_periodic(checkpoint_root: str | Path) -> list[Path]:
    root = Path(checkpoint_root)
    if not root.exists():
        return []
    out = []
    for p in root.iterdir():
        m = re.fullmatch(r"checkpoint_step_(\d+)", p.name)
        if m and (p / META).exists():
            out.append((int(m.group(1)), p))
    return [p for _, p in sorted(out)]


def resolve_resume_path(spec: Optional[str], checkpoint_root: str | Path) -> Optional[Path]:
    if spec is None:
        return None
    if spec == "latest":
        return find_latest_checkpoint(checkpoint_root)
    p = Path(spec)
    if not (p / META).exists():
        raise FileNotFoundError(f"no checkpoint at {p}")
    return p


def cleanup_old_checkpoints(checkpoint_root: str | Path, keep: int) -> list[Path]:
    if keep <= 0:
        return []
    old = list_periodic(checkpoint_root)[:-keep]
    for p in old:
        shutil.rmtree(p, ignore_errors=True)
    return old
