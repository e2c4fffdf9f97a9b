"""Module path of the reference's weight-sync controller (trainer/sglang_controller.py:16).
``SglangController`` is ``EngineController`` (same constructor and ``sync_weights``); against a
real sglang server, which applies commands asynchronously, pass ``settle_s`` to wait between
the protocol's steps."""
from .engine_controller import EngineController

SglangController = EngineController

__all__ = ["SglangController", "EngineController"]
