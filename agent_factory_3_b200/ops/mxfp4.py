"""MXFP4 (OCP microscaling FP4) codec.

Storage layout is the gpt-oss checkpoint layout: ``blocks`` uint8 [..., G, 16] holds 32 E2M1
values per block (low nibble first), ``scales`` uint8 [..., G] holds one E8M0 exponent per block
(value = fp4 * 2^(scale - 127)).  Decode semantics match the reference oracle
``_mxfp4_to_bf16_pytorch`` (models/gpt_oss/quantization.py:102-122 of agent-factory-3).
"""
from __future__ import annotations

import torch

from ._ext import ext, use_cuda_kernels

FP4_VALUES = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
              -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0)


def dequantize_reference(blocks: torch.Tensor, scales: torch.Tensor,
                         dtype=torch.bfloat16) -> torch.Tensor:
    """[..., G, 16] u8 + [..., G] u8 -> [..., G*32] (fp32 math, exact, then cast)."""
    lut = torch.tensor(FP4_VALUES, dtype=torch.float32, device=blocks.device)
    b = blocks.to(torch.int64)
    lo = lut[b & 0xF]
    hi = lut[b >> 4]
    vals = torch.stack([lo, hi], dim=-1).reshape(*blocks.shape[:-1], 32)
    exp = scales.to(torch.int32) - 127
    out = torch.ldexp(vals, exp.unsqueeze(-1).to(torch.float32))
    return out.reshape(*blocks.shape[:-2], blocks.shape[-2] * 32).to(dtype)


def dequantize(blocks: torch.Tensor, scales: torch.Tensor, out: torch.Tensor | None = None):
    """MXFP4 -> bf16 [..., G*32]."""
    if not use_cuda_kernels(blocks, scales):
        r = dequantize_reference(blocks, scales)
        if out is not None:
            out.copy_(r)
            return out
        return r
    if out is None:
        out = torch.empty(*blocks.shape[:-2], blocks.shape[-2] * 32, device=blocks.device,
                          dtype=torch.bfloat16)
    ext().mxfp4_dequant(blocks.contiguous(), scales.contiguous(), out)
    return out


def quantize(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Round-to-nearest MXFP4 quantisation of ``w`` [..., K] (K % 32 == 0).

    The block scale is the smallest power of two that maps the block's absmax into the E2M1
    range (max 6.0); values then round to the nearest representable magnitude.  Used to build
    random-init MXFP4 checkpoints and by tests.
    """
    assert w.shape[-1] % 32 == 0
    x = w.float().reshape(*w.shape[:-1], w.shape[-1] // 32, 32)
    amax = x.abs().amax(dim=-1, keepdim=True).clamp_min(2.0 ** -126)
    e = torch.ceil(torch.log2(amax / 6.0)).clamp(-127, 127)
    scale = torch.pow(2.0, e)
    y = (x / scale).clamp(-6.0, 6.0)
    # nearest E2M1 magnitude {0, .5, 1, 1.5, 2, 3, 4, 6} via the midpoints between them
    mids = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], device=w.device)
    idx = torch.bucketize(y.abs(), mids)
    code = idx + (y < 0).to(idx.dtype) * 8
    code = torch.where(idx == 0, torch.zeros_like(code), code)
    code = code.to(torch.uint8).reshape(*code.shape[:-1], 16, 2)
    blocks = (code[..., 0] | (code[..., 1] << 4)).to(torch.uint8)
    scales = (e.squeeze(-1) + 127).to(torch.uint8)
    return blocks.contiguous(), scales.contiguous()
