"""Rotary position embedding for gpt-oss: NeoX half rotation with YaRN frequency scaling.

Tables follow the YaRN construction (Peng et al., 2023, "YaRN: Efficient Context Window
Extension"): per-dimension blend of interpolated and extrapolated frequencies with a linear
ramp between the beta_fast / beta_slow wavelength boundaries, and cos/sin scaled by the
attention factor 0.1*ln(factor)+1.  gpt-oss uses theta 150000, factor 32, original context
4096, beta_fast 32, beta_slow 1, no truncation.
"""
from __future__ import annotations

import math

import torch

from ._ext import ext, use_cuda_kernels


def rope_tables(head_dim: int, max_pos: int, theta: float, scaling: dict | None = None,
                device=None) -> tuple[torch.Tensor, torch.Tensor]:
    """cos, sin fp32 [max_pos, head_dim/2] with the attention factor folded in."""
    d = head_dim
    inv = 1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.float64) / d))
    attn = 1.0
    if scaling and scaling.get("rope_type", scaling.get("type")) == "yarn":
        factor = float(scaling["factor"])
        orig = float(scaling["original_max_position_embeddings"])
        beta_fast = float(scaling.get("beta_fast", 32.0))
        beta_slow = float(scaling.get("beta_slow", 1.0))
        truncate = bool(scaling.get("truncate", True))

        def corr_dim(n_rot):
            return (d * math.log(orig / (n_rot * 2 * math.pi))) / (2 * math.log(theta))

        low, high = corr_dim(beta_fast), corr_dim(beta_slow)
        if truncate:
            low, high = math.floor(low), math.ceil(high)
        low, high = max(low, 0), min(high, d - 1)
        if low == high:
            high += 0.001
        ramp = ((torch.arange(d // 2, dtype=torch.float64) - low) / (high - low)).clamp(0, 1)
        extrap_w = 1.0 - ramp
        inv = (inv / factor) * (1 - extrap_w) + inv * extrap_w
        attn = scaling.get("attention_factor") or (0.1 * math.log(factor) + 1.0 if factor > 1 else 1.0)
    pos = torch.arange(max_pos, dtype=torch.float64)
    f = torch.outer(pos, inv)
    cos = (f.cos() * attn).float()
    sin = (f.sin() * attn).float()
    if device is not None:
        cos, sin = cos.to(device), sin.to(device)
    return cos, sin


def apply_rope_reference(x: torch.Tensor, pos: torch.Tensor, cos: torch.Tensor,
                         sin: torch.Tensor, inverse: bool = False) -> torch.Tensor:
    """x [T, H, D] -> rotated (fp32 math, cast back)."""
    c = cos[pos.long()][:, None, :]
    s = sin[pos.long()][:, None, :]
    if inverse:
        s = -s
    h = x.shape[-1] // 2
    x1, x2 = x[..., :h].float(), x[..., h:].float()
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1).to(x.dtype)


def apply_rope_(qkv: torch.Tensor, n_rot_heads: int, head_dim: int, pos: torch.Tensor,
                cos: torch.Tensor, sin: torch.Tensor, inverse: bool = False) -> torch.Tensor:
    """In place on the first n_rot_heads heads of each row of qkv [T, n_heads*head_dim]."""
    if not use_cuda_kernels(qkv):
        T = qkv.shape[0]
        v = qkv[:, : n_rot_heads * head_dim].reshape(T, n_rot_heads, head_dim)
        qkv[:, : n_rot_heads * head_dim] = apply_rope_reference(v, pos, cos, sin, inverse).reshape(T, -1)
        return qkv
    ext().rope_apply(qkv, n_rot_heads, head_dim, pos.to(torch.int32).contiguous(), cos, sin, inverse)
    return qkv
