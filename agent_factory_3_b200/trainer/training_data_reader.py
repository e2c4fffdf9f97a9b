"""Reader of the NPZ training-data dumps written by RolloutSaver (reference:
trainer/training_data_reader.py:51-121)."""
from __future__ import annotations

import json
from pathlib import Path
from typing import Iterator

import numpy as np


def load_batch(path: str | Path) -> dict:
    z = np.load(path)
    out = {k: z[k] for k in z.files if k != "metadata"}
    out["metadata"] = json.loads(bytes(z["metadata"]).decode()) if "metadata" in z.files else []
    return out


def iter_samples(path: str | Path) -> Iterator[dict]:
    b = load_batch(path)
    cu = b["cu_seqlens"]
    for i, meta in enumerate(b["metadata"]):
        s, e = int(cu[i]), int(cu[i + 1])
        rec = {"token_ids": b["token_ids"][s:e], "logprobs": b["logprobs"][s:e],
               "completion_mask": b["completion_mask"][s:e], "advantages": b["advantages"][s:e],
               **meta}
        if "routing_indices" in b:
            rec["routing_indices"] = b["routing_indices"][s:e]
        yield rec


def load_all_batches(directory: str | Path) -> list[dict]:
    return [load_batch(p) for p in sorted(Path(directory).glob("batch_*.npz"))]
