"""Clamped SwiGLU of gpt-oss (alpha 1.702, limit 7) over interleaved (gate, up) columns,
as in the reference's K5/K6 kernels (models/gpt_oss/kernels.py:394-582)."""
from __future__ import annotations

import torch

from ._ext import ext, use_cuda_kernels
from .gemm import SWIGLU_ALPHA, SWIGLU_LIMIT, swiglu_reference


def swiglu_fwd(gate_up: torch.Tensor, alpha=SWIGLU_ALPHA, limit=SWIGLU_LIMIT) -> torch.Tensor:
    if not use_cuda_kernels(gate_up):
        return swiglu_reference(gate_up, alpha, limit).to(gate_up.dtype)
    out = torch.empty(*gate_up.shape[:-1], gate_up.shape[-1] // 2, device=gate_up.device,
                      dtype=gate_up.dtype)
    ext().swiglu_fwd(gate_up.contiguous(), out, alpha, limit)
    return out


def swiglu_bwd(gate_up: torch.Tensor, dout: torch.Tensor, alpha=SWIGLU_ALPHA,
               limit=SWIGLU_LIMIT) -> torch.Tensor:
    if not use_cuda_kernels(gate_up):
        gu = gate_up.float().requires_grad_(True)
        with torch.enable_grad():
            h = swiglu_reference(gu, alpha, limit)
            (d,) = torch.autograd.grad(h, gu, dout.float())
        return d.to(gate_up.dtype)
    dgu = torch.empty_like(gate_up)
    ext().swiglu_bwd(gate_up.contiguous(), dout.contiguous(), dgu, alpha, limit)
    return dgu
