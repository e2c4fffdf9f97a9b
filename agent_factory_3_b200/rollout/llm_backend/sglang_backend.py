"""Client of the sglang ``/generate`` HTTP API, served by this package's engine
(``agent_factory_3_b200.engine``) or by an sglang server.

Request: input_ids, sampling_params{max_new_tokens, temperature, top_p, top_k, min_p,
sampling_seed, stop_token_ids}, stream, return_logprob, logprob_start_len, return_entropy,
top_logprobs_num, return_routed_experts, lora_path, extra_key (prefix-cache salt).
Response: output_ids and meta_info{finish_reason, weight_version, output_token_logprobs,
output_top_logprobs, output_token_entropy, routed_experts (base64 int32 [N-1, L, K]),
cached_tokens, completion_tokens, prompt_tokens}; SSE streaming as ``data: {...}`` lines
ending with ``data: [DONE]`` (output_ids may be incremental or cumulative; log-probs are
cumulative).  Contract from the reference client, rollout/llm_backend/sglang_backend.py.
"""
from __future__ import annotations

import asyncio
import base64
import json
from typing import Any, Optional

import aiohttp
import numpy as np

from ..config import RecordConfig, SamplingParams
from .types import GenerationResult


def normalize_finish_reason(fr) -> Optional[str]:
    if fr is None:
        return None
    if isinstance(fr, dict):
        fr = fr.get("type")
    return {"stop": "stop", "length": "length", "abort": "abort", "eos": "stop"}.get(fr, fr)


class SGLangBackend:
    def __init__(self, base_url: str, *, num_layers: Optional[int] = None,
                 num_experts_per_tok: Optional[int] = None, lora_path: Optional[str] = None,
                 cache_salt: Optional[str] = None, timeout: float = 3600.0,
                 connector_limit: int = 64):
        self.base_url = base_url.rstrip("/")
        self.num_layers = num_layers
        self.num_experts_per_tok = num_experts_per_tok
        self.lora_path = lora_path
        self.cache_salt = cache_salt
        self.timeout = aiohttp.ClientTimeout(total=timeout)
        self.connector_limit = connector_limit
        self._session: Optional[aiohttp.ClientSession] = None

    async def _get_session(self) -> aiohttp.ClientSession:
        if self._session is None or self._session.closed:
            self._session = aiohttp.ClientSession(
                timeout=self.timeout,
                connector=aiohttp.TCPConnector(limit=self.connector_limit, keepalive_timeout=60))
        return self._session

    def _sampling(self, s: SamplingParams, max_tokens: int, stop: list[int]) -> dict:
        p: dict[str, Any] = {"max_new_tokens": max_tokens, "temperature": s.temperature,
                             "top_p": s.top_p, "top_k": s.top_k, "stop_token_ids": list(stop),
                             "skip_special_tokens": False, "no_stop_trim": True}
        if s.min_p is not None:
            p["min_p"] = s.min_p
        if s.seed is not None:
            p["sampling_seed"] = s.seed
        return p

    def _payload(self, prompt, max_tokens, stop, sampling, stream, record, routing) -> dict:
        lp = record is not None and (record.logprobs or record.top_logprobs > 0)
        payload = {"input_ids": list(prompt), "sampling_params": self._sampling(sampling, max_tokens, stop),
                   "stream": stream, "return_logprob": lp, "logprob_start_len": len(prompt),
                   "return_entropy": record is not None and record.entropy,
                   "top_logprobs_num": record.top_logprobs if (record and stream) else 0,
                   "return_routed_experts": routing}
        if self.lora_path is not None:
            payload["lora_path"] = self.lora_path
        if self.cache_salt is not None:
            payload["extra_key"] = self.cache_salt
        return payload

    async def generate(self, prompt_tokens, max_tokens, stop_token_ids, sampling, *, stream=False,
                       stop_event: Optional[asyncio.Event] = None,
                       record: Optional[RecordConfig] = None) -> GenerationResult:
        if stream:
            return await self._generate_streaming(prompt_tokens, max_tokens, stop_token_ids,
                                                  sampling, stop_event, record)
        return await self._generate_non_streaming(prompt_tokens, max_tokens, stop_token_ids,
                                                  sampling, record)

    async def _generate_streaming(self, prompt, max_tokens, stop, sampling, stop_event, record):
        payload = self._payload(prompt, max_tokens, stop, sampling, True, record, False)
        session = await self._get_session()
        token_ids: list[int] = []
        finish = None
        last_lp = last_top = last_ent = None
        wv = None
        async with session.post(f"{self.base_url}/generate", json=payload) as resp:
            resp.raise_for_status()
            async for raw in resp.content:
                if stop_event is not None and stop_event.is_set():
                    finish = "abort"
                    break
                line = raw.decode().strip()
                if not line.startswith("data:"):
                    continue
                body = line[5:].strip()
                if body == "[DONE]":
                    break
                chunk = json.loads(body)
                ids = chunk.get("output_ids", [])
                meta = chunk.get("meta_info", {})
                # incremental vs cumulative output_ids: cumulative lists extend what we have
                if len(ids) >= len(token_ids) and ids[:len(token_ids)] == token_ids and meta.get(
                        "completion_tokens", len(ids)) == len(ids):
                    token_ids = list(ids)
                else:
                    token_ids.extend(ids)
                last_lp = meta.get("output_token_logprobs", last_lp)
                last_top = meta.get("output_top_logprobs", last_top)
                last_ent = meta.get("output_token_entropy", last_ent)
                wv = meta.get("weight_version", wv)
                if meta.get("finish_reason") is not None:
                    finish = normalize_finish_reason(meta["finish_reason"])
        logprobs = [x[0] for x in last_lp] if (record and record.logprobs and last_lp) else None
        top = None
        if record and record.top_logprobs > 0 and last_top:
            top = [{int(it[1]): float(it[0]) for it in pos} if pos else {} for pos in last_top]
        ent = last_ent if (record and record.entropy) else None
        if logprobs is not None and len(logprobs) > len(token_ids):
            logprobs = logprobs[:len(token_ids)]
        return GenerationResult(token_ids, finish, logprobs, top, None, None, None, ent, wv)

    async def _generate_non_streaming(self, prompt, max_tokens, stop, sampling, record):
        routing = record is not None and record.routing_indices
        payload = self._payload(prompt, max_tokens, stop, sampling, False, record, routing)
        session = await self._get_session()
        async with session.post(f"{self.base_url}/generate", json=payload) as resp:
            resp.raise_for_status()
            data = await resp.json()
        ids = data["output_ids"]
        meta = data.get("meta_info", {})
        finish = normalize_finish_reason(meta.get("finish_reason"))
        logprobs = entropy = routing_arr = usage = None
        if record is not None and record.logprobs:
            olp = meta.get("output_token_logprobs")
            if olp is None:
                raise RuntimeError("return_logprob=True but the response lacks output_token_logprobs")
            logprobs = [x[0] for x in olp]
            if len(logprobs) != len(ids):
                raise RuntimeError(f"logprobs/tokens length mismatch: {len(logprobs)} vs {len(ids)}")
        if record is not None and record.entropy:
            entropy = meta.get("output_token_entropy")
            if entropy is None or len(entropy) != len(ids):
                raise RuntimeError("return_entropy=True but output_token_entropy is missing or short")
        if routing:
            b64 = meta.get("routed_experts")
            if b64 is None:
                raise RuntimeError("return_routed_experts=True but the response lacks routed_experts")
            routing_arr = self.decode_routing(b64)
        cached = meta.get("cached_tokens")
        if record is not None and record.usage and meta.get("completion_tokens") is not None:
            usage = {"completion_tokens": meta["completion_tokens"]}
            if meta.get("prompt_tokens") is not None:
                usage["prompt_tokens"] = meta["prompt_tokens"]
            if cached is not None:
                usage["cached_tokens"] = cached
        return GenerationResult(ids, finish, logprobs, None, routing_arr, cached, usage, entropy,
                                meta.get("weight_version"))

    def decode_routing(self, b64: str) -> np.ndarray:
        """base64 int32 [N-1, L, K] -> uint8 (expert ids < 256)."""
        if self.num_layers is None or self.num_experts_per_tok is None:
            raise RuntimeError("num_layers and num_experts_per_tok are needed to decode routing")
        flat = np.frombuffer(base64.b64decode(b64), dtype=np.int32)
        per = self.num_layers * self.num_experts_per_tok
        if flat.size % per:
            raise RuntimeError(f"routed_experts size {flat.size} is not a multiple of L*K={per}")
        arr = flat.reshape(-1, self.num_layers, self.num_experts_per_tok)
        if arr.size and (arr.min() < 0 or arr.max() > 254):
            raise RuntimeError("routed expert id out of the uint8 range")
        return arr.astype(np.uint8)

    async def close(self) -> None:
        if self._session is not None and not self._session.closed:
            await self._session.close()
