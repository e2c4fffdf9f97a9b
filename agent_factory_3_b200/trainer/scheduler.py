"""Learning-rate schedules (the Hugging Face ``get_scheduler`` names and formulas: linear,
cosine, cosine_with_restarts, polynomial, constant, constant_with_warmup, inverse_sqrt)."""
from __future__ import annotations

import math

from torch.optim.lr_scheduler import LambdaLR


def get_scheduler(name: str, optimizer, num_warmup_steps: int = 0,
                  num_training_steps: int = 1_000_000, num_cycles: float = 0.5,
                  power: float = 1.0, lr_end: float = 1e-7) -> LambdaLR:
    w = max(0, num_warmup_steps)
    n = max(1, num_training_steps)

    def warm(step):
        return step / max(1, w)

    if name == "constant":
        f = lambda s: 1.0  # noqa: E731
    elif name == "constant_with_warmup":
        f = lambda s: warm(s) if s < w else 1.0  # noqa: E731
    elif name == "linear":
        f = lambda s: warm(s) if s < w else max(0.0, (n - s) / max(1, n - w))  # noqa: E731
    elif name == "cosine":
        def f(s):
            if s < w:
                return warm(s)
            p = (s - w) / max(1, n - w)
            return max(0.0, 0.5 * (1.0 + math.cos(math.pi * num_cycles * 2.0 * p)))
    elif name == "cosine_with_restarts":
        def f(s):
            if s < w:
                return warm(s)
            p = (s - w) / max(1, n - w)
            if p >= 1.0:
                return 0.0
            return max(0.0, 0.5 * (1.0 + math.cos(math.pi * ((num_cycles * p) % 1.0))))
    elif name == "polynomial":
        lr0 = optimizer.defaults["lr"]

        def f(s):
            if s < w:
                return warm(s)
            if s > n:
                return lr_end / lr0
            rem = 1 - (s - w) / (n - w)
            return ((lr0 - lr_end) * rem ** power + lr_end) / lr0
    elif name == "inverse_sqrt":
        shift = w or 10_000

        def f(s):
            if s < w:
                return warm(s)
            return 1.0 / math.sqrt((s + shift - w) / shift)
    else:
        raise ValueError(f"unknown scheduler {name!r}")
    return LambdaLR(optimizer, f)
