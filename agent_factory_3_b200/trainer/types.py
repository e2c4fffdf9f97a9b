"""Core types of the training pipeline (reference: trainer/types.py:10-113).

``TrainingSample`` keeps the reference's field names; sequence fields may be Python lists
or numpy arrays (arrays avoid per-token Python objects for long agentic traces)."""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

import numpy as np
from pydantic import BaseModel, ConfigDict, model_validator


class TrainingSample(BaseModel):
    model_config = ConfigDict(arbitrary_types_allowed=True)

    sample_id: str
    input_ids: Any                      # list[int] | np.ndarray[int32]
    completion_mask: Any                # 1 for generated tokens
    gen_logprobs: Any                   # rollout log-probs (0 for non-generated)
    gen_entropy: Any | None = None
    advantages: Any                     # per-token advantage * completion_mask
    routing_indices: np.ndarray | None = None   # [T, L, K] uint8 (R3)
    oldest_weight_version: int = 0
    weight_version_token_counts: dict[int, int] = {}
    seq_token_count: int = 0
    prompt_token_count: int = 0
    prompt_sequence_count: int = 1
    prompt_id: str = ""
    divisor: float | None = None

    @model_validator(mode="after")
    def _validate_lengths(self) -> "TrainingSample":
        n = len(self.input_ids)
        for name in ("completion_mask", "gen_logprobs", "advantages"):
            if len(getattr(self, name)) != n:
                raise ValueError(f"{name} has length {len(getattr(self, name))}, expected {n}")
        if self.gen_entropy is not None and len(self.gen_entropy) != n:
            raise ValueError("gen_entropy length mismatch")
        if self.routing_indices is not None and self.routing_indices.shape[0] != n:
            raise ValueError("routing_indices must have one row per token")
        return self

    def num_loss_tokens(self) -> int:
        return int(np.asarray(self.completion_mask).sum())

    def __len__(self) -> int:
        return len(self.input_ids)


@dataclass
class ProcessStats:
    total_groups: int = 0
    retained_groups: int = 0
    filtered_all_failed: int = 0
    filtered_all_solved: int = 0
    filtered_zero_loss: int = 0
    filtered_error: int = 0
    total_results: int = 0
    total_samples: int = 0
    reward_mean: float = 0.0
    reward_max: float = 0.0
    reward_min: float = 0.0
    solve_rate: float = 0.0
    reward_component_means: dict[str, float] = field(default_factory=dict)
    end_reason_counts: dict[str, int] = field(default_factory=dict)
    gen_completion_tokens_per_sec: float = 0.0
    gen_rounds_mean: float = 0.0
    gen_rounds_max: int = 0

    def to_metrics_dict(self) -> dict[str, float | int]:
        d = {
            "process/total_groups": self.total_groups,
            "process/retained_groups": self.retained_groups,
            "process/filtered_all_failed": self.filtered_all_failed,
            "process/filtered_all_solved": self.filtered_all_solved,
            "process/filtered_zero_loss": self.filtered_zero_loss,
            "process/filtered_error": self.filtered_error,
            "process/total_results": self.total_results,
            "process/total_samples": self.total_samples,
            "reward/mean": self.reward_mean,
            "reward/max": self.reward_max,
            "reward/min": self.reward_min,
            "reward/solve_rate": self.solve_rate,
            "gen/completion_tokens_per_sec": self.gen_completion_tokens_per_sec,
            "gen/rounds_mean": self.gen_rounds_mean,
            "gen/rounds_max": self.gen_rounds_max,
        }
        for k, v in self.reward_component_means.items():
            d[f"reward_components/{k}"] = v
        total = self.total_results or 1
        for reason, count in self.end_reason_counts.items():
            d[f"gen/end_reason_rate/{reason}"] = count / total
        return d
