"""FP8 (e4m3) expert GEMMs: the ``dequant_dtype="fp8"`` mode of the MoE layer.

The reference's fp8 mode dequantises the MXFP4 experts to fp8 instead of bf16 and quantises the
activations per token (``models/gpt_oss/kernels.py`` K1 / K3 / K4, ``quantizer_config.py``).
Here:

* weights: MXFP4 -> e4m3 with one fp32 scale per expert (``csrc/gemm_fp8.cu``
  ``mxfp4_to_e4m3``; exact for every block within 14 octaves of the expert's largest block
  scale), plus a transposed copy for the backward's dX = dY W (``transpose_u8``);
* activations / gradients: e4m3 with one fp32 scale per row (amax / 448);
* GEMM: tcgen05 ``kind::f8f6f4`` at twice the bf16 tensor rate; the epilogue multiplies by
  row scale x expert scale and then runs the same fused epilogues as the bf16 path (bias,
  clamped SwiGLU, gate weights, SwiGLU backward).

On the CPU every op has a reference built on ``torch.float8_e4m3fn`` with the same rounding
(round to nearest even, saturating at 448).
"""
from __future__ import annotations

import torch

from ._ext import ext, use_cuda_kernels
from .gemm import (EPI_BF16, EPI_ROWSCALE, EPI_SWIGLU, EPI_SWIGLU_BWD, SWIGLU_ALPHA,
                   SWIGLU_LIMIT, _segments, pick_bn, swiglu_reference)

E4M3_MAX = 448.0


def _to_e4m3_bytes(x: torch.Tensor) -> torch.Tensor:
    return x.float().clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn).view(torch.uint8)


def e4m3_to_float(b: torch.Tensor) -> torch.Tensor:
    return b.view(torch.float8_e4m3fn).float()


def quant_rows(x: torch.Tensor, out: torch.Tensor | None = None,
               scale: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """bf16 [M, K] -> (e4m3 bytes [M, K], fp32 scale [M]) with x ~= bytes * scale."""
    M, K = x.shape
    if out is None:
        out = torch.empty(M, K, device=x.device, dtype=torch.uint8)
    if scale is None:
        scale = torch.empty(M, device=x.device, dtype=torch.float32)
    if use_cuda_kernels(x):
        ext().quant_rows_e4m3(x.contiguous() if x.stride(1) != 1 else x, out, scale)
        return out, scale
    amax = x.float().abs().amax(dim=1)
    sc = torch.where(amax > 0, amax / E4M3_MAX, torch.ones_like(amax))
    inv = torch.where(amax > 0, E4M3_MAX / amax, torch.ones_like(amax))
    out.copy_(_to_e4m3_bytes(x.float() * inv[:, None]))
    scale.copy_(sc)
    return out, scale


def mxfp4_to_e4m3(blocks: torch.Tensor, scales: torch.Tensor, out: torch.Tensor | None = None,
                  expert_scale: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """MXFP4 experts [E, N, K/32, 16] (+ e8m0 [E, N, K/32]) -> (e4m3 [E, N, K], fp32 [E])."""
    E, N, G, _ = blocks.shape
    if out is None:
        out = torch.empty(E, N, G * 32, device=blocks.device, dtype=torch.uint8)
    if expert_scale is None:
        expert_scale = torch.empty(E, device=blocks.device, dtype=torch.float32)
    if blocks.is_cuda and use_cuda_kernels(blocks):
        ext().mxfp4_to_e4m3(blocks, scales, out, expert_scale)
        return out, expert_scale
    from . import mxfp4
    smax = scales.reshape(E, -1).int().amax(dim=1)                       # [E]
    w = mxfp4.dequantize(blocks, scales).float()                         # exact values
    factor = torch.pow(2.0, -(smax.float() - 133.0))                     # 2^-(s_max-133)
    out.copy_(_to_e4m3_bytes(w * factor[:, None, None]))
    expert_scale.copy_(torch.pow(2.0, smax.float() - 133.0))
    return out, expert_scale


def transpose_u8(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """[G, R, C] bytes -> [G, C, R]."""
    G, R, C = x.shape
    if out is None:
        out = torch.empty(G, C, R, device=x.device, dtype=torch.uint8)
    if x.is_cuda and use_cuda_kernels(x):
        ext().transpose_u8(x.contiguous(), out)
        return out
    out.copy_(x.transpose(1, 2))
    return out


def grouped_matmul_f8_reference(a, a_scale, b, b_scale, offsets, epilogue="bf16", bias=None,
                                row_scale=None, aux=None, acc_add=None,
                                act_alpha=SWIGLU_ALPHA, act_limit=SWIGLU_LIMIT):
    R = a.shape[0]
    N = b.shape[1]
    af = e4m3_to_float(a) * a_scale.float()[:R, None]
    res = torch.zeros(R, N, dtype=torch.float32, device=a.device)
    for g, (s, e) in enumerate(_segments(offsets)):
        if e <= s:
            continue
        y = (af[s:e] @ e4m3_to_float(b[g]).t()) * float(b_scale[g])
        if acc_add is not None:
            y = y + acc_add[s:e].float()
        if bias is not None:
            y = y + bias[g].float()
        res[s:e] = y
    out2 = None
    if epilogue == "bf16":
        out = res.to(torch.bfloat16)
    elif epilogue == "rowscale":
        out = (res * row_scale.float()[:R, None]).to(torch.bfloat16)
    elif epilogue == "swiglu":
        out2 = res.to(torch.bfloat16)
        out = swiglu_reference(out2.float(), act_alpha, act_limit).to(torch.bfloat16)
    elif epilogue == "swiglu_bwd":
        with torch.enable_grad():
            gu = aux.detach().float().requires_grad_(True)
            h = swiglu_reference(gu, act_alpha, act_limit)
            (dgu,) = torch.autograd.grad(h, gu, res)
        out = dgu.to(torch.bfloat16)
    else:
        raise ValueError(epilogue)
    return out, out2


def grouped_matmul_f8(a: torch.Tensor, a_scale: torch.Tensor, b: torch.Tensor,
                      b_scale: torch.Tensor, offsets: torch.Tensor, *, epilogue: str = "bf16",
                      bias: torch.Tensor | None = None, row_scale: torch.Tensor | None = None,
                      aux: torch.Tensor | None = None, acc_add: torch.Tensor | None = None,
                      save_preact: bool = False, act_alpha: float = SWIGLU_ALPHA,
                      act_limit: float = SWIGLU_LIMIT, bn: int | None = None, band: int = 4):
    """Per-expert GEMM on e4m3 operands: out = epilogue(a_scale[r] * b_scale[g] *
    a[r] @ b[g]^T (+ acc_add) (+ bias_g)).  a: uint8 [R, K] e4m3 (expert-sorted, 128-row padded
    segments), b: uint8 [G, N, K] e4m3.  Epilogues as :func:`ops.gemm.grouped_matmul`.
    Returns (out, out2)."""
    if not use_cuda_kernels(a, b):
        o, o2 = grouped_matmul_f8_reference(a, a_scale, b, b_scale, offsets, epilogue, bias,
                                            row_scale, aux, acc_add, act_alpha, act_limit)
        return o, (o2 if save_preact else None)
    G, N, K = b.shape
    R = a.shape[0]
    epi = {"bf16": EPI_BF16, "rowscale": EPI_ROWSCALE, "swiglu": EPI_SWIGLU,
           "swiglu_bwd": EPI_SWIGLU_BWD}[epilogue]
    cols = N // 2 if epi == EPI_SWIGLU else (2 * N if epi == EPI_SWIGLU_BWD else N)
    out = torch.empty(R, cols, device=a.device, dtype=torch.bfloat16)
    out2 = None
    if epi == EPI_SWIGLU and save_preact:
        out2 = torch.empty(R, N, device=a.device, dtype=torch.bfloat16)
    if bn is None:
        # an e4m3 MMA reads the same 4 KB A tile per instruction as bf16 but finishes in half the
        # time, so narrow tiles become shared-memory bound: N tiles of 192 or 256 (128 only for
        # narrow outputs)
        bn = pick_bn(N, (256, 192) if N >= 192 else (128,))
    ext().gemm_f8(a, b, out, epi, 1, R, N, K, offsets, G, a_scale, b_scale, bias,
                  bias.stride(0) if bias is not None else 0, row_scale, aux, out2, acc_add,
                  1.0, float(act_alpha), float(act_limit), bn, band, 0)
    return out, out2


def matmul_f8(a: torch.Tensor, a_scale: torch.Tensor, b: torch.Tensor, b_scale: torch.Tensor,
              bn: int = 256) -> torch.Tensor:
    """Dense out[M, N] = a_scale[m] * b_scale * (a @ b^T) in bf16 (e4m3 operands [M, K],
    [N, K]; b_scale a one-element fp32 tensor)."""
    M, K = a.shape
    N = b.shape[0]
    if not use_cuda_kernels(a, b):
        y = (e4m3_to_float(a) * a_scale.float()[:, None]) @ e4m3_to_float(b).t()
        return (y * float(b_scale.reshape(-1)[0])).to(torch.bfloat16)
    out = torch.empty(M, N, device=a.device, dtype=torch.bfloat16)
    ext().gemm_f8(a, b, out, EPI_BF16, 0, M, N, K, None, 1, a_scale, b_scale, None, 0, None,
                  None, None, None, 1.0, SWIGLU_ALPHA, SWIGLU_LIMIT, bn, 8, 0)
    return out


__all__ = ["E4M3_MAX", "e4m3_to_float", "grouped_matmul_f8", "matmul_f8", "mxfp4_to_e4m3",
           "quant_rows", "transpose_u8"]
