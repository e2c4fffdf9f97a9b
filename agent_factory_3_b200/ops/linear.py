"""LoRA-adapted linear layer on tcgen05 GEMMs.

    y = x W^T + b + s * (x A^T) B^T          (W frozen bf16, A/B trainable fp32 masters)

Forward runs two kernels: ``xa = s * x A^T`` ([T, r]) and one dual-operand GEMM
``[x | xa] @ [W | B]^T`` with the bias (and optionally a residual) fused in the epilogue.
Backward: ``dx = [dy | s*dy B] @ [W ; A]`` (one dual GEMM), ``dA = (s*dy B)^T x`` and
``dB = dy^T xa`` (weight-gradient GEMMs with both operands MN-major).

Several LoRA branches that share the input (q/k/v of attention) are fused by stacking the A
factors and laying the B factors out block-diagonally.
"""
from __future__ import annotations

import torch

from . import gemm as G


def _bf16(t: torch.Tensor | None) -> torch.Tensor | None:
    return None if t is None else t.to(torch.bfloat16)


def block_diag_b(bs: list[torch.Tensor]) -> torch.Tensor:
    """[sum out_i, sum r_i] block-diagonal matrix from B_i [out_i, r_i]."""
    rows = sum(b.shape[0] for b in bs)
    cols = sum(b.shape[1] for b in bs)
    out = torch.zeros(rows, cols, device=bs[0].device, dtype=bs[0].dtype)
    r0 = c0 = 0
    for b in bs:
        out[r0:r0 + b.shape[0], c0:c0 + b.shape[1]] = b
        r0 += b.shape[0]
        c0 += b.shape[1]
    return out


class LoraLinearFn(torch.autograd.Function):
    """Inputs: x [T, in] bf16, W [out, in] bf16, bias [out] fp32|None, A [R, in] fp32|None,
    B [out, R] fp32|None (R = stacked rank, B block-diagonal for fused branches), residual
    [T, out] bf16|None, scaling s.  W and bias are frozen."""

    @staticmethod
    def forward(ctx, x, W, bias, A, B, residual, s):
        has_lora = A is not None
        xa = None
        if has_lora:
            Ab, Bb = _bf16(A), _bf16(B)
            xa = G.matmul(x, Ab, alpha=s)                       # [T, R]
            y = G.matmul(x, W, bias=bias, residual=residual, a2=xa, b2=Bb)
        else:
            y = G.matmul(x, W, bias=bias, residual=residual)
        ctx.s = s
        ctx.has_lora = has_lora
        ctx.has_residual = residual is not None
        ctx.save_for_backward(x, W, A, B, xa)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, W, A, B, xa = ctx.saved_tensors
        dy = dy.contiguous()
        s = ctx.s
        dA = dB = None
        if ctx.has_lora:
            Ab, Bb = _bf16(A), _bf16(B)
            dyb = G.matmul(dy, Bb, b_layout="kn", alpha=s)        # [T, R] = s * dy B
            dx = G.matmul(dy, W, b_layout="kn", a2=dyb, b2=Ab)    # dy W + dyb A
            if ctx.needs_input_grad[3]:
                dA = G.matmul(dyb, x, a_layout="km", b_layout="kn", out_dtype=torch.float32)
            if ctx.needs_input_grad[4]:
                dB = G.matmul(dy, xa, a_layout="km", b_layout="kn", out_dtype=torch.float32)
        else:
            dx = G.matmul(dy, W, b_layout="kn")
        dres = dy if ctx.has_residual else None
        return dx, None, None, dA, dB, dres, None


@torch.no_grad()
def lora_linear_masked(x, W, bias, A, B, residual, s, row_mask):
    """Inference form for batches that mix adapters: the adapters' factors are stacked along
    the rank (A [sum R_a, in], B [out, sum R_a]) and ``row_mask`` [T, sum R_a] (0/1, bf16) keeps
    each row's own adapter's rank columns, so one dual GEMM applies a different adapter per row:
    y = x W^T + b + ((s x A^T) * mask) B^T (+ residual).  A row whose columns are all zero gets
    the base projection only."""
    xa = G.matmul(x, _bf16(A), alpha=s) * row_mask
    return G.matmul(x, W, bias=bias, residual=residual, a2=xa, b2=_bf16(B))


def lora_linear(x, W, bias=None, A=None, B=None, residual=None, s=1.0):
    return LoraLinearFn.apply(x, W, bias, A, B, residual, s)
