"""Module path of the reference's engine-metrics module (trainer/sglang_metrics.py); the
implementation is ``trainer.engine_metrics`` (``/v1/loads`` schema and the background drainer)."""
from .engine_metrics import (EngineMetricsDrainer, field_names, parse_loads_response,
                             server_id_from_url)

SglangMetricsDrainer = EngineMetricsDrainer

__all__ = ["SglangMetricsDrainer", "EngineMetricsDrainer", "field_names", "parse_loads_response",
           "server_id_from_url"]
