"""Routed-MoE plumbing on the device: routing (top-k or replay), deterministic grouping of
(token, slot) pairs into 128-row padded expert segments, row gather and top-k combine.

The grouping reproduces the reference's stable sort by expert id
(models/gpt_oss/quantization.py:593-636): within an expert, entries keep their flat
(token * K + slot) order.  Segments are padded to multiples of 128 rows so each tcgen05 GEMM
tile belongs to one expert; padding rows are zero and map to token -1.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from ._ext import ext, use_cuda_kernels

PAD = 128
CHUNK = 2048


def capacity(n_entries: int, n_experts: int) -> int:
    """Rows of the sorted buffer needed for n_entries routed entries (worst-case padding)."""
    return n_entries + n_experts * (PAD - 1)


@dataclass
class Routing:
    ids: torch.Tensor          # [T, K] int32 expert ids
    gates: torch.Tensor        # [T, K] fp32 softmax over the chosen logits
    offsets: torch.Tensor      # [E+1] int32 padded segment starts
    counts: torch.Tensor       # [E] int32 entries per expert
    dest: torch.Tensor         # [T*K] int32 sorted row of each entry
    row_src: torch.Tensor      # [R] int32 token of each sorted row (-1 = padding)
    row_gate: torch.Tensor     # [R] fp32 gate of each sorted row
    n_experts: int
    top_k: int

    @property
    def rows(self) -> int:
        return self.row_src.numel()


def route_reference(logits: torch.Tensor, top_k: int, ids: torch.Tensor | None = None):
    """(ids int32 [T,K], gates fp32 [T,K]); ids given -> replay."""
    lf = logits.float()
    if ids is None:
        _, ids = torch.topk(lf, top_k, dim=-1)
    ids = ids.to(torch.int64)
    gates = torch.softmax(torch.take_along_dim(lf, ids, dim=-1), dim=-1)
    return ids.to(torch.int32), gates


def group_reference(ids: torch.Tensor, gates: torch.Tensor, n_experts: int) -> Routing:
    T, K = ids.shape
    flat = ids.reshape(-1).to(torch.int64)
    counts = torch.bincount(flat, minlength=n_experts)[:n_experts]
    padded = (counts + PAD - 1) // PAD * PAD
    offsets = torch.zeros(n_experts + 1, dtype=torch.int64, device=ids.device)
    offsets[1:] = torch.cumsum(padded, 0)
    R = capacity(flat.numel(), n_experts)
    order = torch.sort(flat, stable=True).indices
    starts = torch.zeros(n_experts + 1, dtype=torch.int64, device=ids.device)
    starts[1:] = torch.cumsum(counts, 0)
    rank = torch.empty_like(flat)
    rank[order] = torch.arange(flat.numel(), device=ids.device)
    dest = offsets[flat] + rank - starts[flat]
    row_src = torch.full((R,), -1, dtype=torch.int32, device=ids.device)
    row_gate = torch.zeros(R, dtype=torch.float32, device=ids.device)
    row_src[dest] = (torch.arange(flat.numel(), device=ids.device) // K).to(torch.int32)
    row_gate[dest] = gates.reshape(-1).float()
    return Routing(ids.to(torch.int32), gates.float(), offsets.to(torch.int32),
                   counts.to(torch.int32), dest.to(torch.int32), row_src, row_gate,
                   n_experts, K)


def route(logits: torch.Tensor, top_k: int, n_experts: int,
          replay_ids: torch.Tensor | None = None) -> Routing:
    """Router top-k (or replay of recorded ids) + grouping, without host synchronisation."""
    if replay_ids is not None and not replay_ids.is_cuda and replay_ids.numel():
        # ids still on the host are checked before they index logits and histograms on the
        # device (ids already on the device were checked where they were collated)
        lo, hi = int(replay_ids.min()), int(replay_ids.max())
        if lo < 0 or hi >= n_experts:
            raise ValueError(f"replayed expert id outside [0, {n_experts}): [{lo}, {hi}]")
    if not use_cuda_kernels(logits):
        ids, gates = route_reference(logits, top_k, replay_ids)
        return group_reference(ids, gates, n_experts)
    T = logits.shape[0]
    lf = logits.float().contiguous()
    if replay_ids is not None:
        ids = replay_ids.to(device=logits.device, dtype=torch.int32).reshape(T, top_k).contiguous()
    else:
        ids = torch.empty(T, top_k, device=logits.device, dtype=torch.int32)
    gates = torch.empty(T, top_k, device=logits.device, dtype=torch.float32)
    ext().moe_route(lf, ids, gates, replay_ids is not None)
    n = T * top_k
    R = capacity(n, n_experts)
    dev = logits.device
    offsets = torch.empty(n_experts + 1, device=dev, dtype=torch.int32)
    counts = torch.empty(n_experts, device=dev, dtype=torch.int32)
    dest = torch.empty(n, device=dev, dtype=torch.int32)
    row_src = torch.empty(R, device=dev, dtype=torch.int32)
    row_gate = torch.empty(R, device=dev, dtype=torch.float32)
    scratch = torch.empty(max(1, (n + CHUNK - 1) // CHUNK) * n_experts, device=dev,
                          dtype=torch.int32)
    ext().moe_group(ids, gates, n_experts, offsets, counts, dest, row_src, row_gate, scratch)
    return Routing(ids, gates, offsets, counts, dest, row_src, row_gate, n_experts, top_k)


def gather_rows(x: torch.Tensor, row_src: torch.Tensor, scale: torch.Tensor | None = None,
                out: torch.Tensor | None = None, zero_pad: bool = True) -> torch.Tensor:
    """out[r] = scale[r] * x[row_src[r]]; rows with row_src < 0 (segment padding) are zeroed, or
    with ``zero_pad=False`` left as they are (inference paths that never read them)."""
    R = row_src.numel()
    if not use_cuda_kernels(x):
        idx = row_src.long().clamp_min(0)
        y = x[idx].float()
        if scale is not None:
            y = y * scale.float()[:, None]
        y = torch.where((row_src >= 0)[:, None], y, torch.zeros_like(y)).to(x.dtype)
        if out is not None:
            out.copy_(y)
            return out
        return y
    if out is None:
        out = torch.empty(R, x.shape[1], device=x.device, dtype=x.dtype)
    ext().gather_rows(x, row_src, scale, out, zero_pad)
    return out


def combine_rows(y: torch.Tensor, dest: torch.Tensor, top_k: int,
                 residual: torch.Tensor | None = None,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """out[t] = sum_k y[dest[t*K+k]] (+ residual[t])."""
    T = dest.numel() // top_k
    if not use_cuda_kernels(y):
        d = dest.long().reshape(T, top_k)
        acc = y[d.clamp_min(0)].float()
        acc = torch.where((d >= 0)[..., None], acc, torch.zeros_like(acc)).sum(1)
        if residual is not None:
            acc = acc + residual.float()
        r = acc.to(y.dtype)
        if out is not None:
            out.copy_(r)
            return out
        return r
    if out is None:
        out = torch.empty(T, y.shape[1], device=y.device, dtype=y.dtype)
    ext().combine_rows(y, dest, top_k, residual, out)
    return out
