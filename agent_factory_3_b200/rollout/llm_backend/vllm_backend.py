"""OpenAI-compatible completions client (token-in / token-out through ``prompt`` token ids).
Kept for inference against OpenAI-style servers; training rollouts use the sglang API
(LoopConfig rejects backend='vllm', as the reference does)."""
from __future__ import annotations

import asyncio
from typing import Optional

import aiohttp

from ..config import RecordConfig, SamplingParams
from .types import GenerationResult


class VLLMBackend:
    def __init__(self, base_url: str, model_name: str, timeout: float = 3600.0):
        self.base_url = base_url.rstrip("/")
        self.model_name = model_name
        self.timeout = aiohttp.ClientTimeout(total=timeout)
        self._session: Optional[aiohttp.ClientSession] = None

    async def _get_session(self):
        if self._session is None or self._session.closed:
            self._session = aiohttp.ClientSession(timeout=self.timeout)
        return self._session

    async def generate(self, prompt_tokens, max_tokens, stop_token_ids, sampling: SamplingParams, *,
                       stream=False, stop_event: Optional[asyncio.Event] = None,
                       record: Optional[RecordConfig] = None) -> GenerationResult:
        body = {"model": self.model_name, "prompt": list(prompt_tokens), "max_tokens": max_tokens,
                "temperature": sampling.temperature, "top_p": sampling.top_p,
                "stop_token_ids": list(stop_token_ids), "skip_special_tokens": False,
                "return_tokens_as_token_ids": True,
                "logprobs": 1 if (record and record.logprobs) else None}
        if sampling.top_k and sampling.top_k > 0:
            body["top_k"] = sampling.top_k
        if sampling.seed is not None:
            body["seed"] = sampling.seed
        s = await self._get_session()
        async with s.post(f"{self.base_url}/v1/completions", json=body) as r:
            r.raise_for_status()
            data = await r.json()
        ch = data["choices"][0]
        lp = ch.get("logprobs") or {}
        toks = lp.get("tokens") or []
        ids = [int(t.split(":")[1]) if isinstance(t, str) and t.startswith("token_id:") else int(t)
               for t in toks]
        lps = lp.get("token_logprobs") if record and record.logprobs else None
        usage = data.get("usage")
        return GenerationResult(ids, ch.get("finish_reason"), lps, None, None, None, usage)

    async def close(self):
        if self._session is not None and not self._session.closed:
            await self._session.close()
