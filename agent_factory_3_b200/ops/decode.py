"""Rollout-engine operators: paged decode attention, KV page store/gather and sampling
(CUDA kernels in csrc/decode_attention.cu and csrc/sampling.cu; PyTorch references below)."""
from __future__ import annotations

import math

import torch

from ._ext import ext, use_cuda_kernels


def decode_attention_reference(q, k_pages, v_pages, page_table, seq_lens, sinks, hq, hkv,
                               window=0, scale=None):
    """q [B, Hq, D]; returns [B, Hq*D] fp32."""
    B, _, D = q.shape
    scale = scale or 1.0 / math.sqrt(D)
    P = k_pages.shape[1]
    out = torch.zeros(B, hq, D, dtype=torch.float32, device=q.device)
    rep = hq // hkv
    for b in range(B):
        L = int(seq_lens[b])
        lo = max(0, L - window) if window else 0
        pos = torch.arange(lo, L, device=q.device)
        pages = page_table[b][pos // P].long()
        k = k_pages[pages, pos % P].float()          # [n, Hkv, D]
        v = v_pages[pages, pos % P].float()
        k = k.repeat_interleave(rep, 1).transpose(0, 1)   # [Hq, n, D]
        v = v.repeat_interleave(rep, 1).transpose(0, 1)
        s = (q[b].float()[:, None, :] @ k.transpose(1, 2)).squeeze(1) * scale   # [Hq, n]
        comb = torch.cat([s, sinks.float()[:, None]], dim=1)
        p = torch.softmax(comb, dim=1)[:, :-1]
        out[b] = (p[:, None, :] @ v).squeeze(1)
    return out.reshape(B, hq * D)


def decode_attention(q, k_pages, v_pages, page_table, seq_lens, sinks, hq, hkv, window=0,
                     scale=None, max_seq_len=None, out=None):
    B = q.shape[0]
    D = q.shape[-1] // hq if q.dim() == 2 else q.shape[-1]
    scale = scale or 1.0 / math.sqrt(D)
    if not use_cuda_kernels(q):
        r = decode_attention_reference(q.reshape(B, hq, D), k_pages, v_pages, page_table, seq_lens,
                                       sinks, hq, hkv, window, scale).to(q.dtype)
        if out is not None:
            out.copy_(r)
            return out
        return r
    if out is None:
        out = torch.empty(B, hq * D, device=q.device, dtype=q.dtype)
    msl = max_seq_len if max_seq_len is not None else int(seq_lens.max().item()) if B else 1
    ext().decode_attention(q.reshape(B, -1), k_pages, v_pages, page_table, seq_lens,
                           sinks.float().contiguous(), out, None, hq, hkv, window, scale, msl)
    return out


def kv_store(qkv, k_off, v_off, slots, k_pages, v_pages):
    """k/v of row i of qkv -> page slot slots[i] (slot = page * page_size + offset)."""
    if not use_cuda_kernels(qkv):
        w = k_pages.shape[-1] * k_pages.shape[-2]
        kp = k_pages.view(-1, w)
        vp = v_pages.view(-1, w)
        ok = slots >= 0
        kp[slots[ok].long()] = qkv[ok, k_off:k_off + w]
        vp[slots[ok].long()] = qkv[ok, v_off:v_off + w]
        return
    ext().kv_store(qkv, k_off, v_off, slots.to(torch.int32).contiguous(), k_pages, v_pages)


def kv_gather(qkv, k_off, v_off, slots, k_pages, v_pages):
    if not use_cuda_kernels(qkv):
        w = k_pages.shape[-1] * k_pages.shape[-2]
        ok = slots >= 0
        qkv[ok, k_off:k_off + w] = k_pages.view(-1, w)[slots[ok].long()]
        qkv[ok, v_off:v_off + w] = v_pages.view(-1, w)[slots[ok].long()]
        return
    ext().kv_gather(qkv, k_off, v_off, slots.to(torch.int32).contiguous(), k_pages, v_pages)


def sample_reference(logits, temperature, min_p=None, generator=None):
    """(tokens, logprob under temperature, entropy under temperature)."""
    lf = logits.float()
    T = temperature.float().clamp_min(1e-6)[:, None]
    z = lf / T
    logp = torch.log_softmax(z, dim=-1)
    ent = -(logp.exp() * logp).sum(-1)
    pr = logp.exp()
    if min_p is not None:
        keep = pr >= min_p.float()[:, None] * pr.max(-1, keepdim=True).values
        pr = pr * keep
    greedy = temperature <= 0
    tok = torch.multinomial(pr / pr.sum(-1, keepdim=True), 1, generator=generator).squeeze(-1)
    tok = torch.where(greedy, lf.argmax(-1), tok)
    return tok.to(torch.int32), logp.gather(-1, tok[:, None].long()).squeeze(-1), ent


def sample(logits, temperature, seeds, step, min_p=None):
    if not use_cuda_kernels(logits):
        return sample_reference(logits, temperature, min_p)
    B = logits.shape[0]
    tok = torch.empty(B, device=logits.device, dtype=torch.int32)
    lp = torch.empty(B, device=logits.device, dtype=torch.float32)
    ent = torch.empty(B, device=logits.device, dtype=torch.float32)
    ext().sample_tokens(logits.float().contiguous(), temperature.float().contiguous(),
                        None if min_p is None else min_p.float().contiguous(),
                        seeds.to(torch.int64).contiguous(), int(step), tok, lp, ent)
    return tok, lp, ent
