"""Protocol every generation backend implements (reference: llm_backend/protocol.py:11-48).

stream=True: incremental tokens, stop_event interruption, logprobs/top-k log-probs;
stream=False: also routed experts and usage.  ``record=None`` is inference mode."""
from __future__ import annotations

import asyncio
from typing import Optional, Protocol, runtime_checkable

from ..config import RecordConfig, SamplingParams
from .types import GenerationResult


@runtime_checkable
class LLMBackend(Protocol):
    async def generate(self, prompt_tokens: list[int], max_tokens: int, stop_token_ids: list[int],
                       sampling: SamplingParams, *, stream: bool = False,
                       stop_event: Optional[asyncio.Event] = None,
                       record: Optional[RecordConfig] = None) -> GenerationResult: ...

    async def close(self) -> None: ...
