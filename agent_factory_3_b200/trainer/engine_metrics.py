"""Engine load metrics: the /v1/loads field schema and a background drainer that logs them
(to wandb under ``sglang/<field>/<server>`` with its own step axis, or to the logger)
(reference: trainer/sglang_metrics.py:51-249)."""
from __future__ import annotations

import logging
import math
import queue
import threading
import time
from dataclasses import dataclass
from typing import Any, Callable, Optional
from urllib.parse import urlparse

logger = logging.getLogger(__name__)
NAN = float("nan")


@dataclass(frozen=True)
class Field:
    name: str
    path: tuple[str, ...]


FIELDS: tuple[Field, ...] = (
    Field("throughput", ("gen_throughput",)),
    Field("kv_usage", ("token_usage",)),
    Field("kv_used_tokens", ("num_used_tokens",)),
    Field("kv_cache_gb", ("memory", "kv_cache_gb")),
    Field("cache_hit_rate", ("cache_hit_rate",)),
    Field("spec_accept_length", ("speculative", "accept_length")),
    Field("spec_accept_rate", ("speculative", "accept_rate")),
    Field("queue_running", ("num_running_reqs",)),
    Field("queue_waiting", ("num_waiting_reqs",)),
    Field("queue_paused", ("queues", "paused")),
    Field("queue_retracted", ("queues", "retracted")),
    Field("queue_grammar", ("queues", "grammar")),
    Field("utilization", ("utilization",)),
)


def field_names() -> tuple[str, ...]:
    return tuple(f.name for f in FIELDS)


def _walk(d: Any, path: tuple[str, ...]) -> Any:
    for k in path:
        if not isinstance(d, dict):
            return None
        d = d.get(k)
    return d


def parse_loads_response(data: dict) -> dict[str, float]:
    try:
        load = data["loads"][0]
    except (KeyError, IndexError, TypeError):
        return {}
    if not isinstance(load, dict):
        return {}
    out = {}
    for f in FIELDS:
        v = _walk(load, f.path)
        try:
            out[f.name] = float(v) if v is not None else NAN
        except (TypeError, ValueError):
            out[f.name] = NAN
    return out


def server_id_from_url(url: str) -> str:
    u = urlparse(url)
    return f"{u.hostname}_{u.port}" if u.port else (u.hostname or url)


class EngineMetricsDrainer:
    """Consumes (timestamp, server_url, metrics) tuples from a queue and logs them."""

    def __init__(self, q, log_fn: Optional[Callable[[dict], None]] = None, interval: float = 1.0):
        self.q = q
        self.log_fn = log_fn
        self.interval = interval
        self.seq = 0
        self._stop = threading.Event()
        self._thread: Optional[threading.Thread] = None
        self.last: dict[str, dict[str, float]] = {}

    def _drain_once(self) -> int:
        n = 0
        while True:
            try:
                ts, url, flat = self.q.get_nowait()
            except (queue.Empty, EOFError, OSError):
                break
            sid = server_id_from_url(url)
            self.last[sid] = flat
            rec = {f"sglang/{k}/{sid}": v for k, v in flat.items() if not math.isnan(v)}
            rec["sglang/_seq"] = self.seq
            self.seq += 1
            if self.log_fn is not None:
                try:
                    self.log_fn(rec)
                except Exception:  # noqa: BLE001
                    logger.debug("metrics log failed", exc_info=True)
            n += 1
        return n

    def start(self) -> "EngineMetricsDrainer":
        def run():
            while not self._stop.is_set():
                self._drain_once()
                self._stop.wait(self.interval)
            self._drain_once()

        self._thread = threading.Thread(target=run, daemon=True, name="engine-metrics")
        self._thread.start()
        return self

    def stop(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=5)
