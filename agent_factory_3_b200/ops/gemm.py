"""tcgen05 GEMMs (dense, ragged-M grouped and ragged-K grouped) with fused epilogues.

Layout vocabulary: ``a`` is ``"mk"`` ([M, K] row-major) or ``"km"`` ([K, M]); ``b`` is ``"nk"``
([N, K], i.e. a PyTorch Linear weight) or ``"kn"`` ([K, N]).  All inputs are bf16; the
accumulator is fp32 in tensor memory.

Every function has a PyTorch reference path (``*_reference``) with identical semantics; it
runs on CPU tensors and is the oracle of the GPU tests.
"""
from __future__ import annotations

import math

import torch

from ._ext import ext, use_cuda_kernels

EPI_BF16, EPI_F32, EPI_SWIGLU, EPI_ROWSCALE, EPI_SWIGLU_BWD, EPI_LSE, EPI_LOGPROB_BWD = range(7)
SCHED_PLAIN, SCHED_GROUPED_M, SCHED_GROUPED_K = range(3)

SWIGLU_ALPHA = 1.702
SWIGLU_LIMIT = 7.0


def pick_bn(n: int, allowed=(256, 192, 128, 64, 32)) -> int:
    """Tile width minimising padded columns (ties go to the wider tile)."""
    best, best_waste = None, None
    for bn in allowed:
        waste = math.ceil(n / bn) * bn - n
        if best is None or waste < best_waste:
            best, best_waste = bn, waste
    return best


def _call(a, a_mn, b, b_mn, out, epi, sched, M, N, K, *, offsets=None, num_groups=1, bias=None,
          bias_gstride=0, row_scale=None, aux=None, out2=None, alpha=1.0, beta=0.0,
          act_alpha=SWIGLU_ALPHA, act_limit=SWIGLU_LIMIT, labels=None, vocab_offset=0,
          lse_part=None, label_logit=None, row_stats=None, n_tiles_total=0, bn=256, band=8,
          out_group_stride=0, max_ctas=0, a2=None, b2=None, K2=0, acc_add=None):
    ext().gemm(a, a_mn, b, b_mn, out, epi, sched, M, N, K, offsets, num_groups, bias,
               bias_gstride, row_scale, aux, out2, float(alpha), float(beta), float(act_alpha),
               float(act_limit), labels, vocab_offset, lse_part, label_logit, row_stats,
               n_tiles_total, bn, band, out_group_stride, max_ctas, a2, b2, K2, acc_add)


def _as_mk(a: torch.Tensor, layout: str) -> torch.Tensor:
    return a if layout == "mk" else a.t()


def _as_kn(b: torch.Tensor, layout: str) -> torch.Tensor:
    return b.t() if layout == "nk" else b


# ------------------------------------------------------------------------------------
# dense
# ------------------------------------------------------------------------------------
def matmul_reference(a, b, a_layout="mk", b_layout="nk", bias=None, alpha=1.0, residual=None,
                     out_dtype=torch.bfloat16, accumulate_into=None, a2=None, b2=None):
    y = _as_mk(a, a_layout).float() @ _as_kn(b, b_layout).float()
    if a2 is not None:
        y = y + _as_mk(a2, a_layout).float() @ _as_kn(b2, b_layout).float()
    y = y * alpha
    if bias is not None:
        y = y + bias.float()
    if residual is not None:
        y = y + residual.float()
    if accumulate_into is not None:
        y = y + accumulate_into.float()
    return y.to(out_dtype)


def matmul(a: torch.Tensor, b: torch.Tensor, *, a_layout: str = "mk", b_layout: str = "nk",
           bias: torch.Tensor | None = None, alpha: float = 1.0,
           residual: torch.Tensor | None = None, out_dtype=None,
           out: torch.Tensor | None = None, accumulate: bool = False, bn: int | None = None,
           band: int = 8, a2: torch.Tensor | None = None,
           b2: torch.Tensor | None = None) -> torch.Tensor:
    """C = alpha * (A @ B [+ A2 @ B2]) (+ bias) (+ residual).  ``accumulate`` (fp32 out):
    C += ....  The optional second pair (same layouts) extends the reduction; it carries the
    LoRA branch of an adapted linear layer.  ``out_dtype`` defaults to bf16 (fp32 inputs on
    the reference path keep fp32)."""
    if out_dtype is None:
        out_dtype = out.dtype if out is not None else (
            torch.float32 if a.dtype == torch.float32 else torch.bfloat16)
    if not use_cuda_kernels(a, b):
        acc = out if (accumulate and out is not None) else None
        y = matmul_reference(a, b, a_layout, b_layout, bias, alpha, residual, out_dtype, acc,
                             a2, b2)
        if out is not None:
            out.copy_(y)
            return out
        return y
    a_mn = a_layout == "km"
    b_mn = b_layout == "kn"
    M = a.shape[1] if a_mn else a.shape[0]
    K = a.shape[0] if a_mn else a.shape[1]
    N = b.shape[1] if b_mn else b.shape[0]
    assert (b.shape[0] if b_mn else b.shape[1]) == K, "inner dimensions differ"
    if out is None:
        out = torch.empty(M, N, device=a.device, dtype=out_dtype)
    dual = a2 is not None
    if bn is None:
        if dual:
            allowed = (256, 192) if b_mn else (256, 192, 128)
        elif a_mn:
            allowed = (256, 192, 128, 64)
        elif b_mn:
            allowed = (256, 192, 128, 64)
        else:
            allowed = (256, 192, 128, 64, 32)
        if M <= 128 and N <= 16384 and not dual and not a_mn and not b_mn:
            # one row of tiles (decode-sized M): narrow tiles so the N tiles cover the SMs
            # instead of leaving most of them idle while a few stream all of B
            narrow = [b for b in (32, 64, 128) if b in allowed and math.ceil(N / b) >= 148]
            allowed = (max(narrow),) if narrow else (min(allowed),)
        bn = pick_bn(N, allowed)
    epi = EPI_F32 if out.dtype == torch.float32 else EPI_BF16
    assert residual is None or epi == EPI_BF16
    K2 = 0
    if dual:
        K2 = a2.shape[0] if a_mn else a2.shape[1]
        a2 = a2 if a2.stride(-1) == 1 else a2.contiguous()
        b2 = b2 if b2.stride(-1) == 1 else b2.contiguous()
    _call(a.contiguous() if a.stride(-1) != 1 else a, a_mn,
          b.contiguous() if b.stride(-1) != 1 else b, b_mn, out, epi, SCHED_PLAIN, M, N, K,
          bias=bias, aux=residual, alpha=alpha, beta=1.0 if accumulate else 0.0, bn=bn, band=band,
          a2=a2, b2=b2, K2=K2)
    return out


# ------------------------------------------------------------------------------------
# grouped (ragged M): expert segments of the sorted token buffer
# ------------------------------------------------------------------------------------
def _segments(offsets: torch.Tensor):
    o = offsets.tolist()
    return [(o[g], o[g + 1]) for g in range(len(o) - 1)]


def swiglu_reference(gate_up: torch.Tensor, alpha=SWIGLU_ALPHA, limit=SWIGLU_LIMIT):
    g = gate_up[..., 0::2].float()
    u = gate_up[..., 1::2].float()
    g = g.clamp(max=limit)
    u = u.clamp(min=-limit, max=limit)
    return g * torch.sigmoid(alpha * g) * (u + 1.0)


def grouped_matmul_reference(a, b, offsets, b_layout="nk", epilogue="bf16", bias=None,
                             row_scale=None, aux=None, alpha=1.0, act_alpha=SWIGLU_ALPHA,
                             act_limit=SWIGLU_LIMIT, a2=None, b2=None, acc_add=None):
    """Reference of :func:`grouped_matmul`; returns (out, out2)."""
    R = a.shape[0]
    N = b.shape[1] if b_layout == "nk" else b.shape[2]
    res = torch.zeros(R, N, dtype=torch.float32, device=a.device)
    for g, (s, e) in enumerate(_segments(offsets)):
        if e <= s:
            continue
        w = b[g].float()
        y = a[s:e].float() @ (w.t() if b_layout == "nk" else w)
        if a2 is not None:
            w2 = b2[g].float()
            y = y + a2[s:e].float() @ (w2.t() if b_layout == "nk" else w2)
        y = y * alpha
        if acc_add is not None:
            y = y + acc_add[s:e].float()
        if bias is not None:
            y = y + bias[g].float()
        res[s:e] = y
    out2 = None
    od = torch.float32 if a.dtype == torch.float32 else torch.bfloat16
    if epilogue == "bf16":
        out = res.to(od)
    elif epilogue == "rowscale":
        out = (res * row_scale.float()[:R, None]).to(od)
    elif epilogue == "swiglu":
        out2 = res.to(od)
        out = swiglu_reference(out2.float(), act_alpha, act_limit).to(od)
    elif epilogue == "swiglu_bwd":
        with torch.enable_grad():
            gu = aux.detach().float().requires_grad_(True)
            h = swiglu_reference(gu, act_alpha, act_limit)
            (dgu,) = torch.autograd.grad(h, gu, res)
        out = dgu.to(od)
    else:
        raise ValueError(epilogue)
    return out, out2


def grouped_matmul(a: torch.Tensor, b: torch.Tensor, offsets: torch.Tensor, *,
                   b_layout: str = "nk", epilogue: str = "bf16",
                   bias: torch.Tensor | None = None, row_scale: torch.Tensor | None = None,
                   aux: torch.Tensor | None = None, out: torch.Tensor | None = None,
                   out2: torch.Tensor | None = None, alpha: float = 1.0,
                   act_alpha: float = SWIGLU_ALPHA, act_limit: float = SWIGLU_LIMIT,
                   save_preact: bool = False, bn: int | None = None, band: int = 4,
                   a2: torch.Tensor | None = None, b2: torch.Tensor | None = None,
                   acc_add: torch.Tensor | None = None):
    """Per-expert GEMM over the expert-sorted, 128-row padded activation buffer.

    a: [R, K] sorted rows; b: [G, N, K] ("nk") or [G, K, N] ("kn"); offsets: int32 [G+1]
    padded segment starts.  Epilogues:
      * ``bf16``: out = alpha*a@b_g^T + bias_g
      * ``rowscale``: out = row_scale[r] * (alpha*a@b_g^T + bias_g)   (MoE gate weights)
      * ``swiglu``: columns interleaved (gate, up) -> out = clamped SwiGLU [R, N/2]; with
        ``save_preact`` the raw gate_up is also written to ``out2`` [R, N]
      * ``swiglu_bwd``: acc = dL/dh, aux = raw gate_up [R, 2N] -> out = dL/d(gate_up) [R, 2N]
    ``acc_add`` (bf16 [R, N]) is added to alpha*acc before bias and epilogue: the result of
    another GEMM over the same rows (e.g. an FP8 base product under a bf16 LoRA product).
    Returns (out, out2).
    """
    if not use_cuda_kernels(a, b):
        o, o2 = grouped_matmul_reference(a, b, offsets, b_layout, epilogue, bias, row_scale, aux,
                                         alpha, act_alpha, act_limit, a2, b2, acc_add)
        if out is not None:
            out.copy_(o)
            o = out
        return o, (o2 if save_preact else None)
    G = b.shape[0]
    b_mn = b_layout == "kn"
    K = a.shape[1]
    N = b.shape[2] if b_mn else b.shape[1]
    R = a.shape[0]
    epi = {"bf16": EPI_BF16, "rowscale": EPI_ROWSCALE, "swiglu": EPI_SWIGLU,
           "swiglu_bwd": EPI_SWIGLU_BWD}[epilogue]
    if out is None:
        cols = N // 2 if epi == EPI_SWIGLU else (2 * N if epi == EPI_SWIGLU_BWD else N)
        out = torch.empty(R, cols, device=a.device, dtype=torch.bfloat16)
    if epi == EPI_SWIGLU and save_preact and out2 is None:
        out2 = torch.empty(R, N, device=a.device, dtype=torch.bfloat16)
    dual = a2 is not None
    if bn is None:
        if dual:
            allowed = (256, 192)
        elif N >= 128:
            allowed = (256, 192, 128)
        else:
            allowed = (64,) if b_mn else (32,)
        bn = pick_bn(N, allowed)
    if epi in (EPI_SWIGLU,):
        assert N % 32 == 0
    _call(a, False, b, b_mn, out, epi, SCHED_GROUPED_M, R, N, K, offsets=offsets, num_groups=G,
          bias=bias, bias_gstride=(bias.stride(0) if bias is not None else 0),
          row_scale=row_scale, aux=aux, out2=out2 if epi == EPI_SWIGLU else None, alpha=alpha,
          act_alpha=act_alpha, act_limit=act_limit, bn=bn, band=band, a2=a2, b2=b2,
          K2=(a2.shape[1] if dual else 0), acc_add=acc_add)
    return out, (out2 if epi == EPI_SWIGLU else None)


# ------------------------------------------------------------------------------------
# grouped (ragged K): per-expert weight gradients
# ------------------------------------------------------------------------------------
def grouped_k_matmul_reference(a, b, offsets, alpha=1.0):
    segs = _segments(offsets)
    out = torch.zeros(len(segs), a.shape[1], b.shape[1], dtype=torch.float32, device=a.device)
    for g, (s, e) in enumerate(segs):
        if e > s:
            out[g] = (a[s:e].float().t() @ b[s:e].float()) * alpha
    return out


def grouped_k_matmul(a: torch.Tensor, b: torch.Tensor, offsets: torch.Tensor, *,
                     alpha: float = 1.0, out: torch.Tensor | None = None,
                     bn: int | None = None) -> torch.Tensor:
    """out[g] = alpha * a[seg_g]^T @ b[seg_g]  -> fp32 [G, M, N] with a: [R, M], b: [R, N]."""
    if not use_cuda_kernels(a, b):
        o = grouped_k_matmul_reference(a, b, offsets, alpha)
        if out is not None:
            out.copy_(o)
            return out
        return o
    G = offsets.numel() - 1
    M, N = a.shape[1], b.shape[1]
    if out is None:
        out = torch.zeros(G, M, N, device=a.device, dtype=torch.float32)
    if bn is None:
        bn = pick_bn(N, (256, 192, 128, 64))
    _call(a, True, b, True, out, EPI_F32, SCHED_GROUPED_K, M, N, 0 + a.shape[0], offsets=offsets,
          num_groups=G, alpha=alpha, bn=bn, out_group_stride=M * N)
    return out
