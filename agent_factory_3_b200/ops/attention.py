"""Causal GQA attention with learned per-head sinks and optional sliding window over packed
variable-length sequences (gpt-oss attention, HF ``eager_attention_forward`` semantics:
the sink logit joins the softmax denominator and is then dropped).

Layout: ``qkv`` [T, (Hq + 2*Hkv) * D] bf16 (q heads, then k heads, then v heads, RoPE already
applied), ``cu_seqlens`` int32 [S+1].  Key j is visible from query i of the same sequence iff
j <= i and (window == 0 or i - j < window).

GPU: the sm_100a flash-attention kernels (tcgen05 S = Q K^T and O = P V with TMEM
accumulators) in csrc/attention_sm100.cu.  CPU: the dense per-sequence reference below.
"""
from __future__ import annotations

import math

import torch

from ._ext import ext, use_cuda_kernels


def split_qkv(qkv: torch.Tensor, hq: int, hkv: int, d: int):
    T = qkv.shape[0]
    q = qkv[:, : hq * d].reshape(T, hq, d)
    k = qkv[:, hq * d:(hq + hkv) * d].reshape(T, hkv, d)
    v = qkv[:, (hq + hkv) * d:].reshape(T, hkv, d)
    return q, k, v


def attention_reference(qkv, cu_seqlens, sinks, hq, hkv, d, window=0, scale=None,
                        return_lse=False):
    """Dense fp32 reference.  Returns out [T, Hq*D] (dtype of qkv) and optionally
    lse [Hq, T] (natural log, sink included)."""
    scale = scale if scale is not None else 1.0 / math.sqrt(d)
    q, k, v = split_qkv(qkv, hq, hkv, d)
    T = qkv.shape[0]
    rep = hq // hkv
    out = torch.zeros(T, hq, d, dtype=torch.float32, device=qkv.device)
    lse = torch.zeros(hq, T, dtype=torch.float32, device=qkv.device)
    cu = cu_seqlens.tolist()
    for s, e in zip(cu[:-1], cu[1:]):
        L = e - s
        if L <= 0:
            continue
        qs = q[s:e].float().transpose(0, 1)                              # [Hq, L, D]
        ks = k[s:e].float().transpose(0, 1).repeat_interleave(rep, 0)   # [Hq, L, D]
        vs = v[s:e].float().transpose(0, 1).repeat_interleave(rep, 0)
        sc = qs @ ks.transpose(1, 2) * scale                              # [Hq, L, L]
        i = torch.arange(L, device=qkv.device)
        allowed = i[None, :] <= i[:, None]
        if window:
            allowed &= (i[:, None] - i[None, :]) < window
        sc = sc.masked_fill(~allowed, float("-inf"))
        sink = sinks.float().reshape(hq, 1, 1).expand(hq, L, 1)
        comb = torch.cat([sc, sink], dim=-1)
        lse[:, s:e] = torch.logsumexp(comb, dim=-1)
        p = torch.softmax(comb, dim=-1)[..., :-1]
        out[s:e] = (p @ vs).transpose(0, 1)
    out = out.reshape(T, hq * d).to(qkv.dtype)
    return (out, lse) if return_lse else out


class _AttentionRef(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, sinks, cu_seqlens, hq, hkv, d, window, scale):
        ctx.save_for_backward(qkv, sinks, cu_seqlens)
        ctx.cfg = (hq, hkv, d, window, scale)
        return attention_reference(qkv, cu_seqlens, sinks, hq, hkv, d, window, scale)

    @staticmethod
    def backward(ctx, dout):
        qkv, sinks, cu = ctx.saved_tensors
        hq, hkv, d, window, scale = ctx.cfg
        with torch.enable_grad():
            x = qkv.detach().float().requires_grad_(True)
            sk = sinks.detach().float().requires_grad_(True)
            o = attention_reference(x, cu, sk, hq, hkv, d, window, scale)
            gx, gs = torch.autograd.grad(o, [x, sk], dout.float())
        return gx.to(qkv.dtype), gs.to(sinks.dtype), None, None, None, None, None, None


class AttentionOutputCache:
    """Attention outputs kept from a checkpointed layer's first forward for its recompute.

    Activation checkpointing runs each decoder layer's forward twice.  For full-attention
    layers over long packed sequences the attention kernel dominates that recompute, while
    its result -- O [T, Hq*64] bf16 plus the LSE [Hq, T] fp32 the backward needs anyway -- is
    small next to what checkpointing saves.  Up to ``budget_bytes`` of such results are kept
    (first come, first kept) and handed to the recompute, which then skips the kernel.  Each
    entry is released when the recompute takes it, so its memory lives from the layer's
    forward to the start of the layer's backward."""

    def __init__(self, budget_bytes: int):
        self.budget = int(budget_bytes)
        self.used = 0
        self.entries: dict = {}
        self.hits = 0

    def take(self, key):
        e = self.entries.pop(key, None)
        if e is not None:
            self.used -= e[0].numel() * e[0].element_size() + e[1].numel() * 4
            self.hits += 1
        return e

    def offer(self, key, out, lse) -> None:
        n = out.numel() * out.element_size() + lse.numel() * 4
        if key is None or key in self.entries or self.used + n > self.budget:
            return
        self.entries[key] = (out, lse)
        self.used += n


class _AttentionKernel(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, sinks, cu_seqlens, hq, hkv, d, window, scale, plan, cache_key=None):
        cache = plan.cache if cache_key is not None else None
        hit = cache.take(cache_key) if cache is not None else None
        if hit is not None:   # recompute of a checkpointed layer: reuse the first forward's result
            out, lse = hit
        else:
            out = torch.empty(qkv.shape[0], hq * d, device=qkv.device, dtype=qkv.dtype)
            lse = torch.empty(hq, qkv.shape[0], device=qkv.device, dtype=torch.float32)
            ext().attn_fwd(qkv, sinks.float().contiguous(), plan.tiles, plan.cu, out, lse, hq,
                           hkv, d, window, scale)
            if cache is not None:
                cache.offer(cache_key, out, lse)
        ctx.save_for_backward(qkv, sinks, out, lse)
        ctx.cfg = (hq, hkv, d, window, scale, plan)
        return out

    @staticmethod
    def backward(ctx, dout):
        qkv, sinks, out, lse = ctx.saved_tensors
        hq, hkv, d, window, scale, plan = ctx.cfg
        dqkv = torch.empty_like(qkv)
        dsinks = torch.zeros(hq, device=qkv.device, dtype=torch.float32)
        ext().attn_bwd(qkv, sinks.float().contiguous(), plan.kv_tiles, plan.cu, out,
                       dout.contiguous(), lse, dqkv, dsinks, hq, hkv, d, window, scale)
        return dqkv, dsinks.to(sinks.dtype), None, None, None, None, None, None, None, None


class AttentionPlan:
    """Host-built tile lists for one packed batch (reused by every layer of a step).

    tiles: int32 [n, 3] = (seq_start, q_start, q_end) query spans of up to 256 rows (the
    forward kernel splits each into two 128-row tiles sharing the key blocks), heaviest first;
    kv_tiles: int32 [m, 4] = (seq_start, seq_end, k_start, k_end) key tiles of 128 rows for
    the backward pass, heaviest (most queries after them) first."""

    BLOCK = 128
    SPAN = 256

    def __init__(self, cu_seqlens: torch.Tensor, device):
        cu = [int(x) for x in cu_seqlens.tolist()]
        tiles, kv = [], []
        for s, e in zip(cu[:-1], cu[1:]):
            for q0 in range(s, e, self.SPAN):
                tiles.append((s, q0, min(q0 + self.SPAN, e)))
            for q0 in range(s, e, self.BLOCK):
                kv.append((s, e, q0, min(q0 + self.BLOCK, e)))
        order = sorted(tiles, key=lambda t: -(t[2] - t[0]))  # longest causal prefix first
        self.tiles = torch.tensor(order or [(0, 0, 0)], dtype=torch.int32, device=device)
        kv_order = sorted(kv, key=lambda t: -(t[1] - t[2]))   # most later queries first
        self.kv_tiles = torch.tensor(kv_order or [(0, 0, 0, 0)], dtype=torch.int32, device=device)
        self.cu = torch.tensor(cu, dtype=torch.int32, device=device)
        self.n_tiles = len(tiles)
        self.cache: AttentionOutputCache | None = None   # set by a checkpointed training forward


_HAS_KERNEL = None


def kernel_available() -> bool:
    global _HAS_KERNEL
    if _HAS_KERNEL is None:
        try:
            _HAS_KERNEL = hasattr(ext(), "attn_fwd") and hasattr(ext(), "attn_bwd")
        except RuntimeError:
            _HAS_KERNEL = False
    return _HAS_KERNEL


def attention(qkv: torch.Tensor, sinks: torch.Tensor, cu_seqlens: torch.Tensor, hq: int,
              hkv: int, d: int, window: int = 0, scale: float | None = None,
              plan: AttentionPlan | None = None, cache_key=None) -> torch.Tensor:
    """``cache_key`` (e.g. the layer index) lets a checkpointed layer's recompute reuse the
    output of its first forward when ``plan.cache`` is set (see AttentionOutputCache)."""
    scale = scale if scale is not None else 1.0 / math.sqrt(d)
    if use_cuda_kernels(qkv) and kernel_available() and d == 64:
        if plan is None:
            plan = AttentionPlan(cu_seqlens, qkv.device)
        return _AttentionKernel.apply(qkv, sinks, cu_seqlens, hq, hkv, d, window, scale, plan,
                                      cache_key)
    return _AttentionRef.apply(qkv, sinks, cu_seqlens, hq, hkv, d, window, scale)
