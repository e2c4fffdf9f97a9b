"""Kernel-level comparison against the reference's own GPU kernels on the same B200.

The reference's full training path cannot import offline (it needs ``triton_kernels``,
``accelerate`` and ``peft``), but several of its hot kernels need only ``torch`` and
``triton``.  This benchmark loads those files UNMODIFIED from the reference install
(``baseline/_ref/agent_factory_3/...``) by file path, so no package ``__init__`` with the
missing imports runs, and times them against this library's kernels on the same shapes:

* MXFP4 -> bf16 dequantisation (``models/gpt_oss/kernels.py:206`` ``mxfp4_to_bf16_triton``)
  vs ``mxfp4_dequant``;
* clamped SwiGLU forward / backward (``models/gpt_oss/kernels.py:451`` and ``:556``) vs the
  standalone ``swiglu_fwd`` / ``swiglu_bwd`` kernels (training fuses both into the grouped
  GEMM epilogues, so the fused path has no separate launch at all);
* fused linear -> log-prob / entropy over the 201088-token vocabulary, forward + backward
  (``trainer/losses/linear_cross_entropy.py:39`` ``LinearCrossEntropy``, verl's Triton
  kernels) vs ``linear_logprob_entropy``;
* causal GQA attention, head_dim 64, 64 query / 8 KV heads, forward and backward: torch
  ``flex_attention`` (the reference's B200 attention, ``trainer/training_config.py:24``)
  vs ``attn_fwd`` / ``attn_bwd``.  flex_attention runs without the learned sinks (the
  reference adds them through the HF attention wrapper); the sink costs one extra column.

    python -m agent_factory_3_b200.benchmarks.vs_reference [--ops dequant,swiglu,logprob,attn]

Prints one JSON line per (op, implementation) with the CUDA-event median time.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import math
import os
import sys
import types

import torch

from .kernels import _peaks, _time, attention_flops

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), "..", ".."))
REF = os.path.join(ROOT, "baseline", "_ref", "agent_factory_3")


def _load(relpath: str, name: str, package: str | None = None):
    """Import one reference source file by path (no package __init__ runs)."""
    path = os.path.join(REF, relpath)
    if not os.path.exists(path):
        raise FileNotFoundError(f"reference file missing: {path} (install the reference into "
                                f"baseline/_ref first)")
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    if package:
        mod.__package__ = package
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def _ref_losses_pkg():
    """linear_cross_entropy.py does ``from . import kernels``: give it a bare package that
    holds only the reference's kernels.py, loaded by path."""
    pkg_name = "_af3ref_losses"
    if pkg_name in sys.modules:
        return sys.modules[pkg_name]
    pkg = types.ModuleType(pkg_name)
    pkg.__path__ = [os.path.join(REF, "trainer", "losses")]
    sys.modules[pkg_name] = pkg
    pkg.kernels = _load("trainer/losses/kernels.py", f"{pkg_name}.kernels", pkg_name)
    pkg.linear_cross_entropy = _load("trainer/losses/linear_cross_entropy.py",
                                     f"{pkg_name}.linear_cross_entropy", pkg_name)
    return pkg


def _emit(op, impl, ms, extra):
    print(json.dumps({"op": op, "impl": impl, "ms": round(ms, 4), **extra}), flush=True)


def bench_dequant(iters):
    from ..ops._ext import ext
    ref = _load("models/gpt_oss/kernels.py", "_af3ref_gptoss_kernels")
    E, N, K = 128, 5760, 2880   # gpt-oss-120b gate_up stack of one layer
    blocks = torch.randint(0, 256, (E, N, K // 32, 16), dtype=torch.uint8, device="cuda")
    scales = torch.randint(112, 130, (E, N, K // 32), dtype=torch.uint8, device="cuda")
    out = torch.empty(E, N, K, dtype=torch.bfloat16, device="cuda")
    ext().mxfp4_dequant(blocks, scales, out)
    r = ref.mxfp4_to_bf16_triton(blocks, scales)
    same = bool(torch.equal(r.view(torch.int16), out.view(torch.int16)))
    nbytes = blocks.numel() + scales.numel() + out.numel() * 2
    del r
    ms_ref = _time(lambda: ref.mxfp4_to_bf16_triton(blocks, scales), iters)
    ms_our = _time(lambda: ext().mxfp4_dequant(blocks, scales, out), iters)
    _, hbm, kind = _peaks()
    for impl, ms in (("reference_triton", ms_ref), ("ours", ms_our)):
        gbs = nbytes / (ms / 1e3) / 1e9
        _emit("mxfp4_dequant_120b_gate_up", impl, ms,
              {"gb_per_s": round(gbs, 1), f"frac_of_{kind}_hbm": round(gbs / hbm, 3),
               "bitwise_equal": same})


def bench_swiglu(iters, tokens):
    from ..ops.activation import swiglu_bwd, swiglu_fwd
    ref = _load("models/gpt_oss/kernels.py", "_af3ref_gptoss_kernels")
    M, I = tokens * 4, 2880     # top-4 expert rows, gpt-oss intermediate size
    gu = (torch.randn(M, 2 * I, device="cuda") * 3).bfloat16()
    dout = torch.randn(M, I, device="cuda").bfloat16()
    a, lim = 1.702, 7.0
    h_ref = ref._swiglu_forward_triton(gu, a, lim)
    h_our = swiglu_fwd(gu, a, lim)
    fwd_err = (h_ref.float() - h_our.float()).abs().max().item()
    ms_rf = _time(lambda: ref._swiglu_forward_triton(gu, a, lim), iters)
    ms_of = _time(lambda: swiglu_fwd(gu, a, lim), iters)
    # the reference's backward takes de-interleaved gate / up saved by its forward
    _, gate, up = ref._swiglu_forward_triton(gu, a, lim, save_for_bwd=True)
    d_ref = ref._swiglu_backward(dout, gate, up, a, lim)
    d_our = swiglu_bwd(gu, dout, a, lim)
    # the two differ where an input sits exactly on the clamp limit: the reference's kernel
    # passes no gradient there (strict <), torch's clamp autograd (and this library) does
    tie = torch.stack([gu[:, 0::2] == lim, gu[:, 1::2].abs() == lim], -1).reshape(gu.shape)
    bwd_err = (d_ref.float() - d_our.float()).abs().masked_fill(tie, 0).max().item()
    ties = int(tie.sum())
    ms_rb = _time(lambda: ref._swiglu_backward(dout, gate, up, a, lim), iters)
    ms_ob = _time(lambda: swiglu_bwd(gu, dout, a, lim), iters)
    _, hbm, kind = _peaks()
    fb = gu.numel() * 2 + dout.numel() * 2
    bb = gu.numel() * 2 * 2 + dout.numel() * 2
    for op, impl, ms, nb, err in (("swiglu_fwd", "reference_triton", ms_rf, fb, fwd_err),
                                  ("swiglu_fwd", "ours", ms_of, fb, fwd_err),
                                  ("swiglu_bwd", "reference_triton", ms_rb, bb, bwd_err),
                                  ("swiglu_bwd", "ours", ms_ob, bb, bwd_err)):
        gbs = nb / (ms / 1e3) / 1e9
        _emit(op, impl, ms, {"rows": M, "gb_per_s": round(gbs, 1),
                             f"frac_of_{kind}_hbm": round(gbs / hbm, 3),
                             "max_abs_diff_vs_other": err,
                             **({"limit_ties_excluded": ties} if op == "swiglu_bwd" else {})})


def bench_logprob(iters, tokens):
    from ..ops.logprob import linear_logprob_entropy
    pkg = _ref_losses_pkg()
    T, H, V = tokens, 2880, 201088
    g = torch.Generator(device="cuda").manual_seed(0)
    hidden = (torch.randn(T, H, device="cuda", generator=g) * 0.5).bfloat16().requires_grad_(True)
    weight = (torch.randn(V, H, device="cuda", generator=g) * 0.02).bfloat16()
    labels = torch.randint(0, V, (T,), device="cuda", generator=g)
    glp = torch.randn(T, device="cuda", generator=g)

    def ref_step():
        lp, ent = pkg.linear_cross_entropy.LinearCrossEntropy.apply(hidden, weight, labels, 1.0,
                                                                    "none", None)
        torch.autograd.backward([lp], [glp])
        return lp

    def our_step():
        lp, ent = linear_logprob_entropy(hidden, weight, labels, 1.0)
        torch.autograd.backward([lp], [glp])
        return lp

    lp_r = ref_step().detach()
    lp_o = our_step().detach()
    err = (lp_r.float() - lp_o.float()).abs().max().item()
    hidden.grad = None
    peak, _, kind = _peaks()
    # forward GEMM + backward recompute GEMM + d_hidden GEMM (the reference also computes
    # d_weight, a fourth GEMM that a frozen LM head does not need)
    fl = 3 * 2 * T * V * H
    for impl, fn in (("reference_triton", ref_step), ("ours", our_step)):
        def run():
            hidden.grad = None
            fn()
        ms = _time(run, iters)
        tf = fl / (ms / 1e3) / 1e12
        _emit("linear_logprob_fwd_bwd_201k_vocab", impl, ms,
              {"tokens": T, "tflops_3gemm": round(tf, 1), f"frac_of_{kind}_bf16": round(tf / peak, 3),
               "max_abs_logprob_diff": err})


def bench_attention(iters, seqlen):
    from torch.nn.attention.flex_attention import create_block_mask, flex_attention

    from ..ops import attention as A
    hq, hkv, d = 64, 8, 64
    T = seqlen
    g = torch.Generator(device="cuda").manual_seed(0)
    qkv = torch.randn(T, (hq + 2 * hkv) * d, device="cuda", generator=g).bfloat16()
    sinks = torch.full((hq,), -1e4, device="cuda")   # sinks off, to match flex_attention
    cu = torch.tensor([0, T], dtype=torch.int32)
    plan = A.AttentionPlan(cu, "cuda")
    out = torch.empty(T, hq * d, device="cuda").bfloat16()
    lse = torch.empty(hq, T, device="cuda")
    scale = 1 / math.sqrt(d)
    ext = A.ext()
    dout = torch.randn_like(out)
    dqkv = torch.empty_like(qkv)
    ds = torch.zeros(hq, device="cuda")

    def our_fwd():
        ext.attn_fwd(qkv, sinks, plan.tiles, plan.cu, out, lse, hq, hkv, d, 0, scale)

    def our_bwd():
        ext.attn_bwd(qkv, sinks, plan.kv_tiles, plan.cu, out, dout, lse, dqkv, ds, hq, hkv, d, 0,
                     scale)

    q = qkv[:, : hq * d].view(1, T, hq, d).transpose(1, 2).contiguous().requires_grad_(True)
    k = qkv[:, hq * d:(hq + hkv) * d].view(1, T, hkv, d).transpose(1, 2).contiguous().requires_grad_(True)
    v = qkv[:, (hq + hkv) * d:].view(1, T, hkv, d).transpose(1, 2).contiguous().requires_grad_(True)

    def causal(b, h, qi, ki):
        return qi >= ki

    bm = create_block_mask(causal, 1, 1, T, T, device="cuda")
    flex = torch.compile(flex_attention)   # flex_attention is only fast when compiled
    fo = flex(q, k, v, block_mask=bm, enable_gqa=True, scale=scale)
    our_fwd()
    err = (fo.transpose(1, 2).reshape(T, hq * d).float() - out.float()).abs().max().item()
    gfo = dout.view(1, T, hq, d).transpose(1, 2)

    def flex_fwd():
        with torch.no_grad():
            flex(q, k, v, block_mask=bm, enable_gqa=True, scale=scale)

    def flex_fwd_bwd():
        o = flex(q, k, v, block_mask=bm, enable_gqa=True, scale=scale)
        torch.autograd.backward([o], [gfo])

    ms_ff = _time(flex_fwd, iters)
    ms_ffb = _time(flex_fwd_bwd, iters)
    ms_of = _time(our_fwd, iters)
    ms_ob = _time(our_bwd, iters)
    peak, _, kind = _peaks()
    ff = attention_flops([T], hq, d, 0)
    fb = attention_flops([T], hq, d, 0, bwd=True)
    rows = (("attn_fwd", "reference_flex_attention", ms_ff, ff),
            ("attn_fwd", "ours", ms_of, ff),
            ("attn_bwd", "reference_flex_attention", ms_ffb - ms_ff, fb),
            ("attn_bwd", "ours", ms_ob, fb))
    for op, impl, ms, fl in rows:
        tf = fl / (ms / 1e3) / 1e12
        _emit(f"{op}_causal_{T}_64q8kv_d64", impl, ms,
              {"tflops": round(tf, 1), f"frac_of_{kind}_bf16": round(tf / peak, 3),
               "fwd_max_abs_diff": err,
               **({"note": "flex backward = (fwd+bwd) - fwd"} if impl.startswith("reference")
                  and op == "attn_bwd" else {})})


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ops", default="dequant,swiglu,logprob,attn")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--tokens", type=int, default=16384)
    ap.add_argument("--seqlen", type=int, default=32768)
    args = ap.parse_args()
    torch.cuda.set_device(0)
    for op in args.ops.split(","):
        try:
            if op == "dequant":
                bench_dequant(args.iters)
            elif op == "swiglu":
                bench_swiglu(args.iters, args.tokens)
            elif op == "logprob":
                bench_logprob(args.iters, args.tokens)
            elif op == "attn":
                bench_attention(args.iters, args.seqlen)
            torch.cuda.synchronize()
        except Exception as e:  # noqa: BLE001 - report and go on with the next op
            print(json.dumps({"op": op, "error": f"{type(e).__name__}: {e}"[:400]}), flush=True)
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
