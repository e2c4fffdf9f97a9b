"""Fused linear -> log-prob / entropy over a large vocabulary, without materialising the
[T, V] logits.

Forward: one tcgen05 GEMM ``hidden @ W^T / temperature`` whose epilogue keeps an online
(max, sum exp, sum z*exp) per row over each 256-column vocabulary tile and records the label
logit; a merge kernel combines the tiles into log Z, the entropy H = log Z - E[z] and
logprob = z_label - log Z.

Backward: per vocabulary chunk, the same GEMM recomputes the logits and its epilogue emits
dL/dlogits = (g_lp * (1[v=y] - p_v) - g_H * p_v * (z_v - log Z + H)) / temperature in bf16;
a second GEMM accumulates d_hidden += dlogits @ W_chunk in fp32.  No d_weight is computed (the
LM head is frozen under LoRA), unlike the reference's split-N path
(trainer/losses/kernels.py:1267-1379), which always computes it.

Reference math: trainer/losses/torch_functional.py:20-215 of agent-factory-3 (chunked exact
log-softmax and entropy).
"""
from __future__ import annotations

import math

import torch

from . import gemm as G
from ._ext import ext, use_cuda_kernels

BN = 256


def logprob_entropy_reference(hidden, weight, labels, temperature=1.0):
    logits = hidden.float() @ weight.float().t() / temperature
    logp = torch.log_softmax(logits, dim=-1)
    lp = logp.gather(-1, labels.long().unsqueeze(-1)).squeeze(-1)
    ent = -(logp.exp() * logp).sum(-1)
    return lp, ent


class LinearLogprobFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, hidden, weight, labels, temperature, chunk):
        T, H = hidden.shape
        V = weight.shape[0]
        nt = math.ceil(V / BN)
        dev = hidden.device
        parts = torch.empty(T, nt, 3, device=dev, dtype=torch.float32)
        label_logit = torch.empty(T, device=dev, dtype=torch.float32)
        labels32 = labels.to(torch.int32).contiguous()
        out = torch.empty(1, device=dev, dtype=torch.bfloat16)  # unused by the LSE epilogue
        G._call(hidden, False, weight, False, out, G.EPI_LSE, G.SCHED_PLAIN, T, V, H,
                labels=labels32, lse_part=parts, label_logit=label_logit, n_tiles_total=nt,
                alpha=1.0 / temperature, bn=BN, band=8)
        lp = torch.empty(T, device=dev, dtype=torch.float32)
        ent = torch.empty(T, device=dev, dtype=torch.float32)
        logz = torch.empty(T, device=dev, dtype=torch.float32)
        ext().lse_merge(parts, label_logit, lp, ent, logz)
        ctx.save_for_backward(hidden, weight, labels32, logz, ent)
        ctx.temperature = temperature
        ctx.chunk = chunk
        return lp, ent

    @staticmethod
    def backward(ctx, g_lp, g_ent):
        hidden, weight, labels32, logz, ent = ctx.saved_tensors
        T, H = hidden.shape
        V = weight.shape[0]
        dev = hidden.device
        g_lp = torch.zeros(T, device=dev) if g_lp is None else g_lp.float()
        g_ent = torch.zeros(T, device=dev) if g_ent is None else g_ent.float()
        stats = torch.stack([logz, ent, g_lp, g_ent], dim=1).contiguous()
        dh = torch.zeros(T, H, device=dev, dtype=torch.float32)
        chunk = ctx.chunk
        dz = torch.empty(T, chunk, device=dev, dtype=torch.bfloat16)
        for v0 in range(0, V, chunk):
            v1 = min(V, v0 + chunk)
            w = weight[v0:v1]
            dzc = dz[:, : v1 - v0]
            G._call(hidden, False, w, False, dzc, G.EPI_LOGPROB_BWD, G.SCHED_PLAIN, T, v1 - v0, H,
                    labels=labels32, vocab_offset=v0, row_stats=stats,
                    alpha=1.0 / ctx.temperature, bn=BN, band=8)
            G.matmul(dzc, w, b_layout="kn", out=dh, accumulate=True)
        return dh.to(hidden.dtype), None, None, None, None


class _LogprobRef(torch.autograd.Function):
    @staticmethod
    def forward(ctx, hidden, weight, labels, temperature, chunk):
        ctx.save_for_backward(hidden, weight, labels)
        ctx.temperature = temperature
        ctx.chunk = chunk
        with torch.no_grad():
            out = [logprob_entropy_reference(hidden[i:i + chunk], weight, labels[i:i + chunk],
                                             temperature) for i in range(0, hidden.shape[0], chunk)]
        return torch.cat([o[0] for o in out]), torch.cat([o[1] for o in out])

    @staticmethod
    def backward(ctx, g_lp, g_ent):
        hidden, weight, labels = ctx.saved_tensors
        dh = torch.empty_like(hidden, dtype=torch.float32)
        c = ctx.chunk
        for i in range(0, hidden.shape[0], c):
            with torch.enable_grad():
                h = hidden[i:i + c].detach().float().requires_grad_(True)
                lp, ent = logprob_entropy_reference(h, weight, labels[i:i + c], ctx.temperature)
                loss = 0
                if g_lp is not None:
                    loss = loss + (lp * g_lp[i:i + c]).sum()
                if g_ent is not None:
                    loss = loss + (ent * g_ent[i:i + c]).sum()
                (gh,) = torch.autograd.grad(loss, [h])
            dh[i:i + c] = gh
        return dh.to(hidden.dtype), None, None, None, None


def linear_logprob_entropy_torch(hidden: torch.Tensor, weight: torch.Tensor, labels: torch.Tensor,
                                 temperature: float = 1.0, chunk: int = 512):
    """The chunked PyTorch path of ``linear_logprob_entropy`` on any device (exact log-softmax
    per chunk of rows, manual backward), for cross-checking the fused kernel."""
    return _LogprobRef.apply(hidden, weight, labels, float(temperature), int(chunk))


def linear_logprob_entropy(hidden: torch.Tensor, weight: torch.Tensor, labels: torch.Tensor,
                           temperature: float = 1.0, chunk: int = 16384):
    """(logprob [T] fp32, entropy [T] fp32) of ``labels`` under softmax(hidden W^T / temp)."""
    if use_cuda_kernels(hidden, weight) and hidden.shape[1] % 8 == 0:
        return LinearLogprobFn.apply(hidden.contiguous(), weight, labels, float(temperature),
                                     int(chunk))
    return _LogprobRef.apply(hidden, weight, labels, float(temperature), min(int(chunk), 512))
