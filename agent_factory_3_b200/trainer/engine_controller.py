"""Weight-sync protocol against the rollout engines' HTTP API (reference:
trainer/sglang_controller.py:34-121).

lora mode:   pause(abort) -> unload adapter -> load adapter -> set weight version -> flush ->
             continue
merged mode: pause(abort, or in_place without flush) -> update_weights_from_disk(version) ->
             continue
direct mode: pause(abort) -> write the LoRA tensors straight into each engine's GPU staging
             buffer (CUDA IPC + one NVLink kernel, no files) -> lora_sync/apply(version) ->
             continue (engines on the trainer's machine)
This package's engine applies each call before answering, so no waits are inserted
(``settle_s=0``, the default).  For servers that apply commands asynchronously (sglang), pass
``settle_s`` to sleep between steps; the reference uses fixed sleeps of 5/3/2/1/2 s (LoRA) and
5/3 s or 2/1 s (merged).
"""
from __future__ import annotations

import asyncio
import logging
import time

import aiohttp

logger = logging.getLogger(__name__)


class EngineController:
    def __init__(self, server_urls: list[str], mode: str = "lora", lora_name: str = "policy",
                 flush_cache: bool = True, settle_s: float = 0.0, timeout_s: float = 600.0):
        if mode not in ("lora", "merged", "direct"):
            raise ValueError("mode must be 'lora', 'merged' or 'direct'")
        self._writers: dict = {}
        self.server_urls = list(server_urls)
        self.mode = mode
        self.lora_name = lora_name
        self.flush_cache = flush_cache
        self.settle_s = settle_s
        self.timeout = aiohttp.ClientTimeout(total=timeout_s)
        self.last_sync_s = 0.0

    async def sync_weights(self, weight_path: str, weight_version: str, *, flush: bool = False) -> float:
        """Returns the wall time the sync took (the exposed sync time)."""
        t0 = time.perf_counter()
        if self.mode == "lora":
            await self._sync_lora(weight_path, weight_version)
        else:
            await self._sync_merged(weight_path, weight_version, flush)
        self.last_sync_s = time.perf_counter() - t0
        return self.last_sync_s

    async def sync_direct(self, tensors: dict, weight_version: str) -> float:
        """Direct GPU sync of ``tensors`` (the model's LoRA factors by internal name)."""
        import base64

        from ..parallel.weight_sync import PeerWriter
        t0 = time.perf_counter()
        async with aiohttp.ClientSession(timeout=self.timeout) as s:
            for u in self.server_urls:
                if u not in self._writers:
                    async with s.post(f"{u}/lora_sync/export", json={}) as r:
                        d = await r.json()
                        if not d.get("success"):
                            raise RuntimeError(f"lora_sync/export failed on {u}: {d}")
                        self._writers[u] = PeerWriter(base64.b64decode(d["handle"]))
        await self._call_all("pause_generation", {"mode": "abort"})
        for u in self.server_urls:
            self._writers[u].write(tensors)
        await self._call_all("lora_sync/apply", {"lora_name": self.lora_name,
                                                 "weight_version": weight_version,
                                                 "flush_cache": True})
        await self._call_all("continue_generation", {})
        self.last_sync_s = time.perf_counter() - t0
        return self.last_sync_s

    async def _settle(self, mult: float = 1.0):
        if self.settle_s > 0:
            await asyncio.sleep(self.settle_s * mult)

    async def _sync_lora(self, path: str, version: str):
        await self._call_all("pause_generation", {"mode": "abort"})
        await self._settle(2.5)
        await self._call_all("unload_lora_adapter", {"lora_name": self.lora_name}, ignore_missing=True)
        await self._settle(1.5)
        await self._call_all("load_lora_adapter", {"lora_name": self.lora_name, "lora_path": path})
        await self._settle(1.0)
        await self._call_all("update_weight_version", {"new_version": version})
        await self._settle(0.5)
        await self._call_all("flush_cache", {})
        await self._settle(1.0)
        await self._call_all("continue_generation", {})

    async def _sync_merged(self, path: str, version: str, flush_override: bool):
        flush = self.flush_cache or flush_override
        await self._call_all("pause_generation", {"mode": "abort" if flush else "in_place"})
        await self._settle(2.5 if flush else 1.0)
        await self._call_all("update_weights_from_disk", {"model_path": path, "flush_cache": flush,
                                                          "weight_version": version})
        await self._settle(1.5 if flush else 0.5)
        await self._call_all("continue_generation", {})

    async def _call_all(self, endpoint: str, body: dict, ignore_missing: bool = False):
        async with aiohttp.ClientSession(timeout=self.timeout) as s:
            await asyncio.gather(*(self._call_one(s, u, endpoint, body, ignore_missing)
                                   for u in self.server_urls))

    async def _call_one(self, s, url, endpoint, body, ignore_missing):
        async with s.post(f"{url}/{endpoint}", json=body) as r:
            if r.status != 200:
                text = await r.text()
                if ignore_missing and "does not exist" in text:
                    return
                raise RuntimeError(f"{endpoint} failed on {url}: {r.status} {text}")
