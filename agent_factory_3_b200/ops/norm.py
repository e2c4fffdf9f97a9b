"""RMSNorm forward/backward (HF GptOssRMSNorm semantics: fp32 statistics and weight)."""
from __future__ import annotations

import torch

from ._ext import ext, use_cuda_kernels


def rmsnorm_reference(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    var = xf.pow(2).mean(-1, keepdim=True)
    return (w.float() * (xf * torch.rsqrt(var + eps))).to(x.dtype)


def rmsnorm_fwd(x: torch.Tensor, w: torch.Tensor, eps: float, save_rstd: bool = True):
    """Returns (y, rstd or None)."""
    if not use_cuda_kernels(x):
        y = rmsnorm_reference(x, w, eps)
        rstd = torch.rsqrt(x.float().pow(2).mean(-1) + eps) if save_rstd else None
        return y, rstd
    y = torch.empty_like(x)
    rstd = torch.empty(x.shape[0], device=x.device, dtype=torch.float32) if save_rstd else None
    ext().rmsnorm_fwd(x, w.float().contiguous(), y, rstd, eps)
    return y, rstd


def rmsnorm_bwd(x, w, dy, rstd, dres=None, need_dw=False):
    """Returns (dx (+ dres), dw or None)."""
    if not use_cuda_kernels(x):
        xf = x.float().requires_grad_(True)
        wf = w.float().detach().requires_grad_(need_dw)
        var = xf.pow(2).mean(-1, keepdim=True)
        y = wf * (xf * torch.rsqrt(var + float(_eps_from(x, rstd))))
        grads = torch.autograd.grad(y, [xf, wf] if need_dw else [xf], dy.float())
        dx = grads[0] + (dres.float() if dres is not None else 0)
        return dx.to(x.dtype), (grads[1] if need_dw else None)
    dx = torch.empty_like(x)
    dw = torch.zeros(w.shape, device=x.device, dtype=torch.float32) if need_dw else None
    ext().rmsnorm_bwd(x, w.float().contiguous(), dy, rstd, dres, dx, dw)
    return dx, dw


def _eps_from(x, rstd):
    # recover eps from the saved rstd of the first row: rstd = 1/sqrt(ms + eps)
    ms = x[:1].float().pow(2).mean()
    return float((1.0 / rstd[:1].double() ** 2 - ms.double()).clamp_min(0).item())


class RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps):
        y, rstd = rmsnorm_fwd(x, w, eps)
        ctx.save_for_backward(x, w, rstd)
        ctx.eps = eps
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, rstd = ctx.saved_tensors
        if x.is_cuda:
            dx, dw = rmsnorm_bwd(x, w, dy.contiguous(), rstd, None, ctx.needs_input_grad[1])
        else:
            xf = x.float().requires_grad_(True)
            wf = w.float().detach().requires_grad_(ctx.needs_input_grad[1])
            with torch.enable_grad():
                y = wf * (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + ctx.eps))
                grads = torch.autograd.grad(y, [xf, wf] if ctx.needs_input_grad[1] else [xf],
                                            dy.float())
            dx = grads[0].to(x.dtype)
            dw = grads[1] if ctx.needs_input_grad[1] else None
        return dx, (dw.to(w.dtype) if dw is not None else None), None


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    shape = x.shape
    y = RMSNormFn.apply(x.reshape(-1, shape[-1]), w, eps)
    return y.reshape(shape)
