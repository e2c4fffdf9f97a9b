"""Loss-divisor assignment, staleness filtering and staleness metrics (reference:
trainer/rl_flow.py:75-166)."""
from __future__ import annotations

import logging

from .types import TrainingSample

logger = logging.getLogger(__name__)

AGGREGATION_MODES = {"token-mean", "seq-mean-token-sum", "seq-mean-token-mean",
                     "prompt-mean-token-mean"}


def assign_divisors(samples: list[TrainingSample], mode: str) -> None:
    """Per-sample loss divisor for the aggregation mode (in place)."""
    if mode not in AGGREGATION_MODES:
        raise ValueError(f"Unknown aggregation mode: {mode}")
    for s in samples:
        if mode == "token-mean":
            s.divisor = float(s.seq_token_count)
        elif mode == "seq-mean-token-sum":
            s.divisor = float(s.prompt_sequence_count)
        elif mode == "seq-mean-token-mean":
            s.divisor = float(s.prompt_sequence_count * s.seq_token_count)
        else:
            s.divisor = float(s.prompt_token_count)


def filter_stale_samples(samples: list[TrainingSample], current_step: int,
                         max_staleness: int) -> list[TrainingSample]:
    """Drop samples whose oldest generating weight version is more than max_staleness steps
    behind current_step (max_staleness < 0 disables the filter)."""
    if max_staleness < 0:
        return samples
    threshold = current_step - max_staleness
    kept = [s for s in samples if s.oldest_weight_version >= threshold]
    if len(kept) != len(samples):
        logger.info("staleness filter dropped %d/%d samples (threshold=%d)",
                    len(samples) - len(kept), len(samples), threshold)
    return kept


def compute_staleness_metrics(samples: list[TrainingSample], current_step: int,
                              pre_filter_count: int) -> tuple[dict[str, float], dict[int, float]]:
    drop = pre_filter_count - len(samples)
    metrics = {"flow/stale_drop_count": float(drop),
               "flow/stale_drop_rate": drop / max(pre_filter_count, 1)}
    version_pct: dict[int, float] = {}
    by_version: dict[int, int] = {}
    for s in samples:
        for v, c in s.weight_version_token_counts.items():
            by_version[v] = by_version.get(v, 0) + c
    total = sum(by_version.values())
    if not samples or total == 0:
        metrics["flow/staleness_mean"] = 0.0
        metrics["flow/staleness_max"] = 0.0
        return metrics, version_pct
    wsum, smax = 0.0, 0
    for v, c in by_version.items():
        st = current_step - v
        pct = c / total
        metrics[f"flow/token_pct/staleness_{st}"] = pct
        version_pct[v] = pct
        wsum += st * c
        smax = max(smax, st)
    metrics["flow/staleness_mean"] = wsum / total
    metrics["flow/staleness_max"] = float(smax)
    return metrics, version_pct
