"""Paged KV cache with page-granular prefix caching.

Pages hold ``page_size`` consecutive tokens of one sequence for every layer (K and V pools
[layers][pages, page_size, Hkv, D] bf16) plus the MoE expert ids chosen for those tokens
([pages, page_size, L, K] uint8, 255 = unknown), so routed experts can be returned for tokens
served from the prefix cache.  Full pages are indexed by a hash chain over their tokens,
salted with the request's cache key and LoRA adapter; cached pages with no owner are kept in
LRU order and reclaimed when the free list runs dry.
"""
from __future__ import annotations

import hashlib
from collections import OrderedDict

import numpy as np
import torch


class OutOfPages(RuntimeError):
    pass


class PagedKVCache:
    @staticmethod
    def bytes_per_page(num_layers: int, page_size: int, hkv: int, head_dim: int, top_k: int,
                       elem_bytes: int = 2) -> int:
        """Device bytes one page holds: K and V of every layer plus the routed-expert capture."""
        return num_layers * page_size * (2 * hkv * head_dim * elem_bytes + top_k)

    @staticmethod
    def pages_for_memory_fraction(fraction: float, total_bytes: int, used_bytes: int,
                                  page_bytes: int) -> int:
        """Pages that fit when this process may use ``fraction`` of the device's memory and
        ``used_bytes`` are taken already (weights, workspaces): the sglang
        ``--mem-fraction-static`` rule, applied to the KV pool."""
        if not 0.0 < fraction <= 1.0:
            raise ValueError(f"memory fraction must be in (0, 1], got {fraction}")
        pages = int((fraction * total_bytes - used_bytes) // page_bytes)
        if pages < 1:
            raise ValueError(f"no room for the KV cache: {fraction:g} of {total_bytes / 2**30:.1f} "
                             f"GiB is below the {used_bytes / 2**30:.1f} GiB already in use")
        return pages

    def __init__(self, num_layers: int, num_pages: int, page_size: int, hkv: int, head_dim: int,
                 top_k: int, device, dtype=torch.bfloat16):
        self.num_layers, self.num_pages, self.page_size = num_layers, num_pages, page_size
        self.hkv, self.head_dim, self.top_k = hkv, head_dim, top_k
        self.device = torch.device(device)
        self.k = [torch.zeros(num_pages, page_size, hkv, head_dim, device=device, dtype=dtype)
                  for _ in range(num_layers)]
        self.v = [torch.zeros(num_pages, page_size, hkv, head_dim, device=device, dtype=dtype)
                  for _ in range(num_layers)]
        self.routing = torch.full((num_pages, page_size, num_layers, top_k), 255, dtype=torch.uint8,
                                  device=device)
        self.refcount = np.zeros(num_pages, dtype=np.int32)
        self.free = list(range(num_pages - 1, -1, -1))
        self.hash_to_page: dict[bytes, int] = {}
        self.page_hash: dict[int, bytes] = {}
        self.lru: OrderedDict[int, None] = OrderedDict()   # cached pages with refcount 0
        self.hits = 0
        self.lookups = 0

    # ------------------------------------------------------------------ accounting
    @property
    def bytes_per_token(self) -> int:
        return self.num_layers * 2 * self.hkv * self.head_dim * 2

    def used_pages(self) -> int:
        return self.num_pages - len(self.free) - len(self.lru)

    def usage(self) -> float:
        return self.used_pages() / self.num_pages

    def gb(self) -> float:
        return self.num_pages * self.page_size * self.bytes_per_token / 1e9

    # ------------------------------------------------------------------ hashing
    @staticmethod
    def chain(prev: bytes, tokens, salt: str) -> bytes:
        h = hashlib.blake2b(digest_size=16)
        h.update(prev)
        h.update(salt.encode())
        h.update(np.asarray(tokens, dtype=np.int64).tobytes())
        return h.digest()

    # ------------------------------------------------------------------ alloc / free
    def _take(self) -> int:
        if self.free:
            p = self.free.pop()
        elif self.lru:
            p, _ = self.lru.popitem(last=False)
            h = self.page_hash.pop(p)
            self.hash_to_page.pop(h, None)
        else:
            raise OutOfPages("KV cache is full")
        self.refcount[p] = 1
        self.routing[p].fill_(255)
        return p

    def can_allocate(self, n_pages: int) -> bool:
        return len(self.free) + len(self.lru) >= n_pages

    def match_prefix(self, tokens: list[int], salt: str) -> tuple[list[int], list[bytes]]:
        """Pages holding the longest cached full-page prefix (refcounts taken)."""
        pages, hashes = [], []
        prev = b""
        P = self.page_size
        n_full = len(tokens) // P
        self.lookups += n_full
        for i in range(n_full):
            h = self.chain(prev, tokens[i * P:(i + 1) * P], salt)
            p = self.hash_to_page.get(h)
            if p is None:
                break
            if self.refcount[p] == 0:
                self.lru.pop(p, None)
            self.refcount[p] += 1
            pages.append(p)
            hashes.append(h)
            prev = h
            self.hits += 1
        return pages, hashes

    def allocate(self, n: int) -> list[int]:
        if not self.can_allocate(n):
            raise OutOfPages(f"need {n} pages")
        return [self._take() for _ in range(n)]

    def register(self, page: int, h: bytes) -> None:
        if h in self.hash_to_page or page in self.page_hash:
            return
        self.hash_to_page[h] = page
        self.page_hash[page] = h

    def release(self, pages: list[int]) -> None:
        for p in pages:
            self.refcount[p] -= 1
            if self.refcount[p] == 0:
                if p in self.page_hash:
                    self.lru[p] = None
                else:
                    self.free.append(p)

    def flush(self) -> None:
        """Drop every cached (unowned) page from the prefix index."""
        for p in list(self.lru.keys()):
            h = self.page_hash.pop(p)
            self.hash_to_page.pop(h, None)
            self.free.append(p)
        self.lru.clear()
        for p, h in list(self.page_hash.items()):
            self.hash_to_page.pop(h, None)
        self.page_hash.clear()

    def cache_hit_rate(self) -> float:
        return self.hits / max(1, self.lookups)
