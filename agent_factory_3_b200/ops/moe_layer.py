"""Routed MoE MLP of gpt-oss with frozen MXFP4 experts and optional per-expert LoRA.

Forward (one token batch, T tokens, top-K):
  logits = x Wr^T + br                         tcgen05 GEMM, fp32 out
  ids, gates = top-K(logits) or replay ids     softmax over the K chosen logits
  grouping -> 128-row padded expert segments   (deterministic, stable by token order)
  x_s = gather(x)                              [R, H]
  [xa]  = s * x_s A_gu_e^T                     LoRA down-projection, [R, r]
  h, gu = SwiGLU([x_s | xa] [W_gu_e | B_gu_e]^T + b_gu_e)     one grouped GEMM, fused epilogue
  [ha]  = s * h A_dn_e^T
  y_s   = gate * ([h | ha] [W_dn_e | B_dn_e]^T + b_dn_e)       one grouped GEMM, fused gates
  out   = residual + sum_k y_s[dest[t, k]]     combine

Backward computes dx and the LoRA gradients only (experts and router are frozen).  As in the
reference (models/gpt_oss/quantization.py:376-421), no gradient flows into the gate weights
or router logits, and the expert weights are re-derived from the MXFP4 bytes instead of being
saved.
"""
from __future__ import annotations

import os

import torch

from . import gemm as G
from . import moe as M
from . import mxfp4
from ._ext import ext, use_cuda_kernels


class ExpertWeights:
    """Frozen MXFP4 expert projections of one layer (uint8 blocks/scales, fp32 biases).

    ``dequantized()`` materialises bf16 [E, N, K] into a scratch buffer shared by all layers
    of the same shape (one layer's MoE runs at a time on the compute stream)."""

    _scratch: dict = {}

    def __init__(self, gu_blocks, gu_scales, gu_bias, dn_blocks, dn_scales, dn_bias, shards=None,
                 dequant_dtype: str = "bf16"):
        self.gu_blocks, self.gu_scales, self.gu_bias = gu_blocks, gu_scales, gu_bias
        self.dn_blocks, self.dn_scales, self.dn_bias = dn_blocks, dn_scales, dn_bias
        # parallel.fsdp.ExpertShards when the blocks / scales above are only this rank's
        # experts; the full stack is then gathered (fused with the dequantisation) on use
        self.shards = shards
        # "bf16": training GEMMs on bf16 dequantised experts; "fp8": e4m3 experts with one
        # scale per expert, e4m3 activations with one scale per row (ops/fp8.py)
        if dequant_dtype not in ("bf16", "fp8"):
            raise ValueError(f"dequant_dtype must be 'bf16' or 'fp8', got {dequant_dtype!r}")
        if dequant_dtype == "fp8" and shards is not None:
            raise ValueError("the fp8 expert mode is not available with sharded experts")
        self.dequant_dtype = dequant_dtype

    @classmethod
    def _buf(cls, key, shape, device, dtype=torch.bfloat16):
        k = (key, tuple(shape), str(device), dtype)
        b = cls._scratch.get(k)
        if b is None:
            b = torch.empty(shape, device=device, dtype=dtype)
            cls._scratch[k] = b
        return b

    def _e4m3(self, which: str, blocks, scales, transposed: bool):
        """(e4m3 [E, N, K] -- or [E, K, N] when ``transposed`` --, fp32 scale [E])."""
        from . import fp8
        E, N, Gk, _ = blocks.shape
        dev = blocks.device
        cuda = blocks.is_cuda
        w = self._buf(which + "8", (E, N, Gk * 32), dev, torch.uint8) if cuda else None
        sc = self._buf(which + "8s", (E,), dev, torch.float32) if cuda else None
        w, sc = fp8.mxfp4_to_e4m3(blocks, scales, out=w, expert_scale=sc)
        if not transposed:
            return w, sc
        wt = self._buf(which + "8t", (E, Gk * 32, N), dev, torch.uint8) if cuda else None
        return fp8.transpose_u8(w, out=wt), sc

    def gate_up_e4m3(self, transposed: bool = False):
        return self._e4m3("gu", self.gu_blocks, self.gu_scales, transposed)

    def down_e4m3(self, transposed: bool = False):
        return self._e4m3("dn", self.dn_blocks, self.dn_scales, transposed)

    def _dequantized(self, which: str, blocks, scales) -> torch.Tensor:
        E, N, Gk, _ = self.shards.shapes[which + "_blocks"] if self.shards else blocks.shape
        out = self._buf(which, (E, N, Gk * 32), blocks.device) if blocks.is_cuda else None
        if self.shards is not None:
            return self.shards.dequantized(which, blocks, scales, out)
        return mxfp4.dequantize(blocks, scales, out=out)

    def gate_up(self) -> torch.Tensor:
        return self._dequantized("gu", self.gu_blocks, self.gu_scales)

    def down(self) -> torch.Tensor:
        return self._dequantized("dn", self.dn_blocks, self.dn_scales)

    @classmethod
    def release_scratch(cls):
        cls._scratch.clear()

    _f16_ok: dict = {}
    _int_ok: dict = {}

    def int_cvt_ok(self) -> bool:
        """True when every block scale s is <= 128 (cached per tensor version)."""
        ok = True
        for sc in (self.gu_scales, self.dn_scales):
            key = (sc.data_ptr(), sc._version, sc.numel())
            v = self._int_ok.get(key)
            if v is None:
                v = bool((sc <= 128).all())
                self._int_ok[key] = v
            ok = ok and v
        return ok

    def f16_exact(self) -> bool:
        """True when every block scale s lies in [104, 140]: then each e2m1 value times
        2^(s-127) is an exact f16 number and the MXFP4-direct kernel (which runs its tile in
        f16) computes the same products as the bf16 dequantised weights.  Cached per tensor
        version, so an in-place weight update is re-checked."""
        ok = True
        for sc in (self.gu_scales, self.dn_scales):
            key = (sc.data_ptr(), sc._version, sc.numel())
            v = self._f16_ok.get(key)
            if v is None:
                v = bool(((sc >= 104) & (sc <= 140)).all())
                self._f16_ok[key] = v
            ok = ok and v
        return ok


def _b(t):
    return None if t is None else t.to(torch.bfloat16)


def _sorted_mask(row_mask: torch.Tensor, rt) -> torch.Tensor:
    """Per-token LoRA rank mask [T, R] -> per expert-sorted row (padding rows zero)."""
    src = rt.row_src.long()
    m = row_mask.index_select(0, src.clamp(min=0))
    return m * (src >= 0).to(m.dtype)[:, None]


def mxfp4_int_cvt(experts: ExpertWeights) -> int:
    """1 to run the MXFP4-direct kernel's integer e2m1 -> f16 conversion (AF3_MXFP4_CVT=int and
    every scale byte <= 128).  The default is the hardware conversion instruction, measured
    faster on B200 (1.95 vs 1.62 TB/s for a 120b MoE layer at 128 tokens)."""
    if os.environ.get("AF3_MXFP4_CVT") != "int":
        return 0
    return 1 if experts.int_cvt_ok() else 0


class MoEFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, xn, residual, router_w, router_b, gu_A, gu_B, dn_A, dn_B, experts,
                top_k, replay_ids, s, act_alpha, act_limit, routing_out, lora_row_mask=None):
        T, H = xn.shape
        E = router_w.shape[0]
        logits = G.matmul(xn, router_w, bias=router_b, out_dtype=torch.float32)
        rt = M.route(logits, top_k, E, replay_ids=replay_ids)
        if routing_out is not None:
            routing_out.append(rt.ids)
        x_s = M.gather_rows(xn, rt.row_src)
        lora_gu = gu_A is not None
        lora_dn = dn_A is not None
        need_grad = torch.is_grad_enabled() or any(ctx.needs_input_grad)
        if experts.dequant_dtype == "fp8":
            return MoEFn._forward_fp8(ctx, xn, residual, rt, x_s, gu_A, gu_B, dn_A, dn_B, experts,
                                      top_k, s, act_alpha, act_limit, need_grad)
        W_gu = experts.gate_up()
        xa = G.grouped_matmul(x_s, _b(gu_A), rt.offsets, alpha=s)[0] if lora_gu else None
        sm = _sorted_mask(lora_row_mask, rt) if lora_row_mask is not None else None
        if sm is not None and xa is not None:
            xa = xa * sm
        h, gu = G.grouped_matmul(x_s, W_gu, rt.offsets, epilogue="swiglu", bias=experts.gu_bias,
                                 act_alpha=act_alpha, act_limit=act_limit,
                                 save_preact=need_grad, a2=xa,
                                 b2=_b(gu_B) if lora_gu else None)
        W_dn = experts.down()
        ha = G.grouped_matmul(h, _b(dn_A), rt.offsets, alpha=s)[0] if lora_dn else None
        if sm is not None and ha is not None:
            ha = ha * sm
        y_s, _ = G.grouped_matmul(h, W_dn, rt.offsets, epilogue="rowscale", bias=experts.dn_bias,
                                  row_scale=rt.row_gate, a2=ha,
                                  b2=_b(dn_B) if lora_dn else None)
        out = M.combine_rows(y_s, rt.dest, top_k, residual=residual)
        ctx.experts = experts
        ctx.cfg = (top_k, s, act_alpha, act_limit, lora_gu, lora_dn)
        ctx.rt = rt
        ctx.save_for_backward(xn, gu_A, gu_B, dn_A, dn_B, xa, h, ha, gu)
        return out

    @staticmethod
    def _forward_fp8(ctx, xn, residual, rt, x_s, gu_A, gu_B, dn_A, dn_B, experts, top_k, s,
                     act_alpha, act_limit, need_grad):
        """Expert GEMMs on e4m3 operands.  The LoRA branches stay bf16 and run as a second
        GEMM over the same rows that adds the e4m3 base product (``acc_add``) before the fused
        epilogue."""
        from . import fp8
        lora_gu, lora_dn = gu_A is not None, dn_A is not None
        x_q, x_sc = fp8.quant_rows(x_s)
        W_gu, s_gu = experts.gate_up_e4m3()
        xa = G.grouped_matmul(x_s, _b(gu_A), rt.offsets, alpha=s)[0] if lora_gu else None
        if lora_gu:
            base, _ = fp8.grouped_matmul_f8(x_q, x_sc, W_gu, s_gu, rt.offsets,
                                            bias=experts.gu_bias)
            h, gu = G.grouped_matmul(xa, _b(gu_B), rt.offsets, epilogue="swiglu",
                                     act_alpha=act_alpha, act_limit=act_limit,
                                     save_preact=need_grad, acc_add=base)
            del base
        else:
            h, gu = fp8.grouped_matmul_f8(x_q, x_sc, W_gu, s_gu, rt.offsets, epilogue="swiglu",
                                          bias=experts.gu_bias, act_alpha=act_alpha,
                                          act_limit=act_limit, save_preact=need_grad)
        del x_q
        h_q, h_sc = fp8.quant_rows(h)
        W_dn, s_dn = experts.down_e4m3()
        ha = G.grouped_matmul(h, _b(dn_A), rt.offsets, alpha=s)[0] if lora_dn else None
        if lora_dn:
            base, _ = fp8.grouped_matmul_f8(h_q, h_sc, W_dn, s_dn, rt.offsets,
                                            bias=experts.dn_bias)
            y_s, _ = G.grouped_matmul(ha, _b(dn_B), rt.offsets, epilogue="rowscale",
                                      row_scale=rt.row_gate, acc_add=base)
            del base
        else:
            y_s, _ = fp8.grouped_matmul_f8(h_q, h_sc, W_dn, s_dn, rt.offsets, epilogue="rowscale",
                                           bias=experts.dn_bias, row_scale=rt.row_gate)
        out = M.combine_rows(y_s, rt.dest, top_k, residual=residual)
        ctx.experts = experts
        ctx.cfg = (top_k, s, act_alpha, act_limit, lora_gu, lora_dn)
        ctx.rt = rt
        ctx.save_for_backward(xn, gu_A, gu_B, dn_A, dn_B, xa, h, ha, gu)
        return out

    @staticmethod
    def _backward_fp8(ctx, dout):
        from . import fp8
        xn, gu_A, gu_B, dn_A, dn_B, xa, h, ha, gu = ctx.saved_tensors
        top_k, s, act_alpha, act_limit, lora_gu, lora_dn = ctx.cfg
        rt = ctx.rt
        experts = ctx.experts
        dout = dout.contiguous()
        g = M.gather_rows(dout, rt.row_src, rt.row_gate)            # gate * dout, [R, H]
        g_q, g_sc = fp8.quant_rows(g)
        W_dnT, s_dn = experts.down_e4m3(transposed=True)            # [E, I, H]: dh = g W_dn
        d_dnA = d_dnB = d_guA = d_guB = None
        if lora_dn:
            gd = G.grouped_matmul(g, _b(dn_B), rt.offsets, b_layout="kn", alpha=s)[0]  # [R, r]
            base, _ = fp8.grouped_matmul_f8(g_q, g_sc, W_dnT, s_dn, rt.offsets)
            dgu, _ = G.grouped_matmul(gd, _b(dn_A), rt.offsets, b_layout="kn",
                                      epilogue="swiglu_bwd", aux=gu, act_alpha=act_alpha,
                                      act_limit=act_limit, acc_add=base)
            del base
            d_dnA = G.grouped_k_matmul(gd, h, rt.offsets)                   # [E, r, I]
            d_dnB = G.grouped_k_matmul(g, ha, rt.offsets)                   # [E, H, r]
        else:
            dgu, _ = fp8.grouped_matmul_f8(g_q, g_sc, W_dnT, s_dn, rt.offsets,
                                           epilogue="swiglu_bwd", aux=gu, act_alpha=act_alpha,
                                           act_limit=act_limit)
        del g, g_q
        d_q, d_sc = fp8.quant_rows(dgu)
        W_guT, s_gu = experts.gate_up_e4m3(transposed=True)         # [E, H, 2I]: dx = dgu W_gu
        if lora_gu:
            ga = G.grouped_matmul(dgu, _b(gu_B), rt.offsets, b_layout="kn", alpha=s)[0]
            base, _ = fp8.grouped_matmul_f8(d_q, d_sc, W_guT, s_gu, rt.offsets)
            dx_s, _ = G.grouped_matmul(ga, _b(gu_A), rt.offsets, b_layout="kn", acc_add=base)
            del base
            x_s = M.gather_rows(xn, rt.row_src)
            d_guA = G.grouped_k_matmul(ga, x_s, rt.offsets)                 # [E, r, H]
            d_guB = G.grouped_k_matmul(dgu, xa, rt.offsets)                 # [E, 2I, r]
        else:
            dx_s, _ = fp8.grouped_matmul_f8(d_q, d_sc, W_guT, s_gu, rt.offsets)
        dxn = M.combine_rows(dx_s, rt.dest, top_k)
        return (dxn, dout, None, None, d_guA, d_guB, d_dnA, d_dnB, None, None, None, None, None,
                None, None, None)

    @staticmethod
    def backward(ctx, dout):
        if ctx.experts.dequant_dtype == "fp8":
            return MoEFn._backward_fp8(ctx, dout)
        xn, gu_A, gu_B, dn_A, dn_B, xa, h, ha, gu = ctx.saved_tensors
        top_k, s, act_alpha, act_limit, lora_gu, lora_dn = ctx.cfg
        rt = ctx.rt
        experts = ctx.experts
        dout = dout.contiguous()
        g = M.gather_rows(dout, rt.row_src, rt.row_gate)            # gate * dout, [R, H]
        W_dn = experts.down()                                       # [E, H, I] = (K=H, N=I)
        d_dnA = d_dnB = d_guA = d_guB = None
        if lora_dn:
            gd = G.grouped_matmul(g, _b(dn_B), rt.offsets, b_layout="kn", alpha=s)[0]  # [R, r]
            dgu, _ = G.grouped_matmul(g, W_dn, rt.offsets, b_layout="kn", epilogue="swiglu_bwd",
                                      aux=gu, act_alpha=act_alpha, act_limit=act_limit,
                                      a2=gd, b2=_b(dn_A))
            d_dnA = G.grouped_k_matmul(gd, h, rt.offsets)                   # [E, r, I]
            d_dnB = G.grouped_k_matmul(g, ha, rt.offsets)                   # [E, H, r]
        else:
            dgu, _ = G.grouped_matmul(g, W_dn, rt.offsets, b_layout="kn", epilogue="swiglu_bwd",
                                      aux=gu, act_alpha=act_alpha, act_limit=act_limit)
        del g
        W_gu = experts.gate_up()                                    # [E, 2I, H] = (K=2I, N=H)
        if lora_gu:
            ga = G.grouped_matmul(dgu, _b(gu_B), rt.offsets, b_layout="kn", alpha=s)[0]
            dx_s, _ = G.grouped_matmul(dgu, W_gu, rt.offsets, b_layout="kn", a2=ga,
                                       b2=_b(gu_A))
            x_s = M.gather_rows(xn, rt.row_src)
            d_guA = G.grouped_k_matmul(ga, x_s, rt.offsets)                 # [E, r, H]
            d_guB = G.grouped_k_matmul(dgu, xa, rt.offsets)                 # [E, 2I, r]
        else:
            dx_s, _ = G.grouped_matmul(dgu, W_gu, rt.offsets, b_layout="kn")
        dxn = M.combine_rows(dx_s, rt.dest, top_k)
        return (dxn, dout, None, None, d_guA, d_guB, d_dnA, d_dnB, None, None, None, None, None,
                None, None, None)


def _mxfp4_direct(xn: torch.Tensor, experts: ExpertWeights, E: int, top_k: int) -> bool:
    """Inference with few rows per expert and f16-exact scales: run the experts on the MXFP4
    bytes directly.  AF3_MOE_MXFP4=0/1 forces the choice (the scale check still applies)."""
    if (not xn.is_cuda or not use_cuda_kernels(xn) or experts.shards is not None
            or not experts.f16_exact()):
        return False
    flag = os.environ.get("AF3_MOE_MXFP4")
    if flag is not None:
        return flag == "1"
    if torch.is_grad_enabled():
        return False
    return xn.shape[0] * top_k <= 128 * E


def _token_tile(rows: int, E: int) -> int:
    avg = rows / max(1, E)
    return 16 if avg <= 12 else 32 if avg <= 28 else 64 if avg <= 56 else 128


def moe_forward_mxfp4(xn, residual, router_w, router_b, experts: ExpertWeights, top_k: int,
                      lora: dict | None = None, s: float = 1.0, replay_ids=None,
                      act_alpha: float = 1.702, act_limit: float = 7.0,
                      routing_out: list | None = None, lora_row_mask=None):
    """Inference MoE that reads the MXFP4 expert weights directly (no bf16 copy): the
    swap-AB kernel tiles 128 weight rows x the few tokens of each expert, and expert LoRA
    (x A_e^T s) B_e^T joins the same accumulation as extra K blocks."""
    lora = lora or {}
    T, H = xn.shape
    E = router_w.shape[0]
    logits = G.matmul(xn, router_w, bias=router_b, out_dtype=torch.float32)
    rt = M.route(logits, top_k, E, replay_ids=replay_ids)
    if routing_out is not None:
        routing_out.append(rt.ids)
    x_s = M.gather_rows(xn, rt.row_src, zero_pad=False)   # padding rows are never read
    R = x_s.shape[0]
    bn = _token_tile(T * top_k, E)
    I2 = experts.gu_blocks.shape[1]
    gu_A, gu_B, dn_A, dn_B = (lora.get(k) for k in ("gu_A", "gu_B", "dn_A", "dn_B"))
    xa = G.grouped_matmul(x_s, _b(gu_A), rt.offsets, alpha=s)[0] if gu_A is not None else None
    sm = _sorted_mask(lora_row_mask, rt) if lora_row_mask is not None else None
    if sm is not None and xa is not None:
        xa = xa * sm
    h = torch.empty(R, I2 // 2, device=xn.device, dtype=torch.bfloat16)
    ic = mxfp4_int_cvt(experts)
    ext().moe_mxfp4_gemm(x_s, experts.gu_blocks, experts.gu_scales, experts.gu_bias, rt.offsets,
                         rt.counts, 0, None, h, act_alpha, act_limit, bn,
                         lora_b=_b(gu_B) if xa is not None else None, xa=xa, int_cvt=ic)
    ha = G.grouped_matmul(h, _b(dn_A), rt.offsets, alpha=s)[0] if dn_A is not None else None
    if sm is not None and ha is not None:
        ha = ha * sm
    y_s = torch.empty(R, H, device=xn.device, dtype=torch.bfloat16)
    ext().moe_mxfp4_gemm(h, experts.dn_blocks, experts.dn_scales, experts.dn_bias, rt.offsets,
                         rt.counts, 1, rt.row_gate, y_s, act_alpha, act_limit, bn,
                         lora_b=_b(dn_B) if ha is not None else None, xa=ha, int_cvt=ic)
    return M.combine_rows(y_s, rt.dest, top_k, residual=residual)


def moe_forward(xn, residual, router_w, router_b, experts: ExpertWeights, top_k: int,
                lora: dict | None = None, s: float = 1.0, replay_ids=None,
                act_alpha: float = 1.702, act_limit: float = 7.0, routing_out: list | None = None,
                lora_row_mask: torch.Tensor | None = None):
    """``lora_row_mask`` [T, R] (0/1): per-token selection of expert-LoRA rank columns when
    ``lora`` holds several adapters stacked along the rank (mixed-adapter inference batches);
    the gate_up and down factors must use the same column layout."""
    lora = lora or {}
    if _mxfp4_direct(xn, experts, router_w.shape[0], top_k):
        return moe_forward_mxfp4(xn, residual, router_w, router_b, experts, top_k, lora, s,
                                 replay_ids, act_alpha, act_limit, routing_out, lora_row_mask)
    return MoEFn.apply(xn, residual, router_w, router_b, lora.get("gu_A"), lora.get("gu_B"),
                       lora.get("dn_A"), lora.get("dn_B"), experts, top_k, replay_ids, s,
                       act_alpha, act_limit, routing_out, lora_row_mask)
