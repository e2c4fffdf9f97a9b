"""Progress and throughput of a batch of rollouts (tqdm when attached to a terminal)."""
from __future__ import annotations

import time
from collections import Counter

from .config import RolloutResult


class ExecutionMonitor:
    def __init__(self, total: int, desc: str = "rollouts", use_tqdm: bool = True):
        self.total = total
        self.start = time.time()
        self.done = 0
        self.success = 0
        self.tokens = 0
        self.end_reasons: Counter = Counter()
        self._bar = None
        if use_tqdm:
            try:
                from tqdm import tqdm
                self._bar = tqdm(total=total, desc=desc, leave=False)
            except Exception:  # noqa: BLE001
                self._bar = None

    def update(self, r: RolloutResult) -> None:
        self.done += 1
        self.success += int(r.is_task_success)
        self.tokens += r.num_generated_tokens
        self.end_reasons[r.end_reason or "failed"] += 1
        if self._bar is not None:
            self._bar.update(1)
            self._bar.set_postfix(ok=self.success, tok_s=f"{self.tokens_per_sec():.0f}")

    def tokens_per_sec(self) -> float:
        return self.tokens / max(1e-6, time.time() - self.start)

    def summary(self) -> dict:
        el = time.time() - self.start
        return {"total": self.total, "done": self.done, "success": self.success,
                "success_rate": self.success / max(1, self.done), "generated_tokens": self.tokens,
                "tokens_per_sec": self.tokens / max(1e-6, el), "elapsed": el,
                "end_reasons": dict(self.end_reasons)}

    def close(self) -> None:
        if self._bar is not None:
            self._bar.close()
