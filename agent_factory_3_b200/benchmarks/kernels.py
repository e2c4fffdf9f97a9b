"""Micro-benchmarks of the sm_100a kernels, timed with CUDA events after warm-up.

    python -m agent_factory_3_b200.benchmarks.kernels --op attn_fwd --seqlens 8192 --iters 10
    python -m agent_factory_3_b200.benchmarks.kernels --op attn_bwd --seqlens 8192
    python -m agent_factory_3_b200.benchmarks.kernels --op gemm --m 16384 --n 5760 --k 2880
    python -m agent_factory_3_b200.benchmarks.kernels --op moe --tokens 32768
    python -m agent_factory_3_b200.benchmarks.kernels --op dequant --experts 128
    python -m agent_factory_3_b200.benchmarks.kernels --op moe_decode --tokens 128 --path mxfp4
    python -m agent_factory_3_b200.benchmarks.kernels --op decode_attn --tokens 128 --seqlens 1024

Each run prints one JSON line with the time per call, the achieved TFLOP/s (or GB/s) and the
fraction of the measured peak in MEASURED_PEAKS.json (when present).
"""
from __future__ import annotations

import argparse
import json
import math
import os

import torch


def _peaks():
    p = os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return d.get("bf16_tflops", 1590.0), d.get("hbm_gbs", 6650.0), "measured"
    except OSError:
        return 1590.0, 6650.0, "fallback"


def _time(fn, iters, warmup=3, flush_bytes=0):
    flush = torch.empty(flush_bytes // 4, dtype=torch.float32, device="cuda") if flush_bytes else None
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        if flush is not None:
            flush.zero_()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    times.sort()
    return times[len(times) // 2]


def attention_flops(seqlens, hq, d, window, bwd=False):
    f = 0
    for L in seqlens:
        if window:
            pairs = sum(min(i + 1, window) for i in range(L))
        else:
            pairs = L * (L + 1) // 2
        f += 4 * pairs * d * hq
    return f * (2.5 if bwd else 1.0)


def bench_attention(args, bwd):
    from ..ops import attention as A
    hq, hkv, d = args.hq, args.hkv, 64
    seqlens = [int(x) for x in args.seqlens.split(",")]
    T = sum(seqlens)
    qkv = torch.randn(T, (hq + 2 * hkv) * d, device="cuda").bfloat16()
    sinks = torch.randn(hq, device="cuda")
    cu = torch.tensor([0] + torch.tensor(seqlens).cumsum(0).tolist(), dtype=torch.int32)
    plan = A.AttentionPlan(cu, "cuda")
    out = torch.empty(T, hq * d, device="cuda").bfloat16()
    lse = torch.empty(hq, T, device="cuda")
    scale = 1 / math.sqrt(d)
    ext = A.ext()

    def fwd():
        ext.attn_fwd(qkv, sinks, plan.tiles, plan.cu, out, lse, hq, hkv, d, args.window, scale)

    if not bwd:
        ms = _time(fwd, args.iters)
    else:
        fwd()
        dout = torch.randn_like(out)
        dqkv = torch.empty_like(qkv)
        ds = torch.zeros(hq, device="cuda")

        def b():
            ext.attn_bwd(qkv, sinks, plan.kv_tiles, plan.cu, out, dout, lse, dqkv, ds, hq, hkv, d,
                         args.window, scale)

        ms = _time(b, args.iters)
    fl = attention_flops(seqlens, hq, d, args.window, bwd)
    return {"flops": fl, "ms": ms}


def bench_gemm(args):
    from ..ops import gemm as G
    a = torch.randn(args.m, args.k, device="cuda").bfloat16()
    b = torch.randn(args.n, args.k, device="cuda").bfloat16()
    if getattr(args, "dtype", "bf16") == "fp8":
        from ..ops import fp8
        aq, asc = fp8.quant_rows(a)
        bq, _ = fp8.quant_rows(b)
        one = torch.ones(1, device="cuda")
        ms = _time(lambda: fp8.matmul_f8(aq, asc, bq, one), args.iters)
        return {"flops": 2 * args.m * args.n * args.k, "ms": ms}
    out = torch.empty(args.m, args.n, device="cuda").bfloat16()
    ms = _time(lambda: G.matmul(a, b, out=out), args.iters)
    return {"flops": 2 * args.m * args.n * args.k, "ms": ms}


def bench_moe(args):
    from ..ops import moe as M
    from ..ops import gemm as G
    E, K, H, I = 128, 4, 2880, 2880
    T = args.tokens
    logits = torch.randn(T, E, device="cuda")
    rt = M.route(logits, K, E)
    x = torch.randn(T, H, device="cuda").bfloat16()
    xs = M.gather_rows(x, rt.row_src)
    W = (torch.randn(E, 2 * I, H, device="cuda") * 0.02).bfloat16()
    bias = torch.zeros(E, 2 * I, device="cuda")
    if getattr(args, "dtype", "bf16") == "fp8":
        # e4m3 operands (kind::f8f6f4): the GEMM alone, operands quantised once outside
        from ..ops import fp8
        xq, xsc = fp8.quant_rows(xs)
        Wq, _ = fp8.quant_rows(W.reshape(E * 2 * I, H))
        Wq = Wq.reshape(E, 2 * I, H)
        es = torch.ones(E, device="cuda")
        ms = _time(lambda: fp8.grouped_matmul_f8(xq, xsc, Wq, es, rt.offsets, epilogue="swiglu",
                                                 bias=bias), args.iters)
        return {"flops": 2 * T * K * 2 * I * H, "ms": ms}
    ms = _time(lambda: G.grouped_matmul(xs, W, rt.offsets, epilogue="swiglu", bias=bias), args.iters)
    return {"flops": 2 * T * K * 2 * I * H, "ms": ms}


def bench_dequant(args):
    """MXFP4 -> bf16 of one gpt-oss-120b gate_up expert stack [E, 5760, 2880]."""
    from ..ops._ext import ext
    E, N, K = args.experts, 5760, 2880
    blocks = torch.randint(0, 256, (E, N, K // 32, 16), dtype=torch.uint8, device="cuda")
    scales = torch.randint(112, 130, (E, N, K // 32), dtype=torch.uint8, device="cuda")
    out = torch.empty(E, N, K, dtype=torch.bfloat16, device="cuda")
    ms = _time(lambda: ext().mxfp4_dequant(blocks, scales, out), args.iters)
    return {"bytes": blocks.numel() + scales.numel() + out.numel() * 2, "ms": ms}


def bench_decode_attn(args):
    """Paged decode attention: ``--tokens`` sequences of ``--seqlens`` cached tokens each (64-token
    pages, scattered), one query token per sequence; bytes = K and V read once."""
    from ..ops import decode as D
    B, L, hq, hkv, d, P = args.tokens, int(args.seqlens.split(",")[0]), args.hq, args.hkv, 64, 64
    npg = (L + P - 1) // P
    g = torch.Generator(device="cuda").manual_seed(0)
    kp = torch.randn(B * npg + 1, P, hkv, d, device="cuda", generator=g).bfloat16()
    vp = torch.randn_like(kp)
    perm = torch.randperm(B * npg, device="cuda", generator=g).to(torch.int32)
    pt = perm.view(B, npg)
    lens = torch.full((B,), L, device="cuda", dtype=torch.int32)
    q = torch.randn(B, hq * d, device="cuda", generator=g).bfloat16()
    sinks = torch.zeros(hq, device="cuda")
    out = torch.empty_like(q)
    ms = _time(lambda: D.decode_attention(q, kp, vp, pt, lens, sinks, hq, hkv, args.window, None, L,
                                          out=out), args.iters, flush_bytes=256 << 20)
    return {"bytes": 2 * B * L * hkv * d * 2, "ms": ms}


def bench_moe_decode(args):
    """One gpt-oss-120b MoE layer (128 experts, top-4, H = I = 2880) at decode batch sizes:
    the MXFP4-direct path (AF3_MOE_MXFP4=1) or the dequantise + grouped GEMM path (=0).
    Bytes = MXFP4 weights of the experts that received tokens (the roofline of decode)."""
    from ..ops import mxfp4
    from ..ops.moe_layer import ExpertWeights, moe_forward
    E, K, H, I = 128, 4, 2880, 2880
    T = args.tokens
    g = torch.Generator(device="cuda").manual_seed(0)
    gu_b = torch.randint(0, 256, (E, 2 * I, H // 32, 16), device="cuda", dtype=torch.uint8, generator=g)
    gu_s = torch.randint(118, 124, (E, 2 * I, H // 32), device="cuda", dtype=torch.uint8, generator=g)
    dn_b = torch.randint(0, 256, (E, H, I // 32, 16), device="cuda", dtype=torch.uint8, generator=g)
    dn_s = torch.randint(118, 124, (E, H, I // 32), device="cuda", dtype=torch.uint8, generator=g)
    ex = ExpertWeights(gu_b, gu_s, torch.zeros(E, 2 * I, device="cuda"), dn_b, dn_s,
                       torch.zeros(E, H, device="cuda"))
    router_w = torch.randn(E, H, device="cuda").bfloat16()
    router_b = torch.zeros(E, device="cuda")
    xn = torch.randn(T, H, device="cuda").bfloat16()
    os.environ["AF3_MOE_MXFP4"] = "1" if args.path == "mxfp4" else "0"
    with torch.no_grad():
        logits = xn.float() @ router_w.float().t()
        hit = torch.unique(logits.topk(K, -1).indices).numel()
        ms = _time(lambda: moe_forward(xn, xn, router_w, router_b, ex, K), args.iters,
                   flush_bytes=256 << 20)
    per_expert = (2 * I * H + H * I) * 17 // 32   # e2m1 nibbles + one scale byte per 32
    return {"bytes": hit * per_expert, "ms": ms, "experts_hit": hit}


def bench_peer_sync(args):
    """Fused fp32 -> bf16 cast + NVLink store of LoRA-sized tensors from GPU 0 into a staging
    buffer on GPU 1 (the direct trainer -> engine weight sync).  Bytes = bf16 bytes stored."""
    from ..parallel.weight_sync import PeerWriter, StagingBuffer
    if torch.cuda.device_count() < 2:
        raise SystemExit("peer_sync needs two GPUs")
    n_tensors = 64
    per = (args.tokens * 1024) // n_tensors // 8 * 8      # --tokens = total MElements
    shapes = {f"t{i}": (per,) for i in range(n_tensors)}
    st = StagingBuffer.for_tensors(shapes, "cuda:1")
    torch.cuda.set_device(0)
    src = {k: torch.randn(*v, device="cuda:0") for k, v in shapes.items()}
    w = PeerWriter(st)
    ms = _time(lambda: w.write(src, stream_sync=False), args.iters)
    ok = bool(torch.equal(st.tensors()["t3"].cpu(), src["t3"].bfloat16().cpu()))
    return {"bytes": per * n_tensors * 2, "ms": ms, "correct": ok}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--dtype", choices=["bf16", "fp8"], default="bf16",
                    help="operand type of the GEMM (--op gemm / moe)")
    ap.add_argument("--op", required=True, choices=["attn_fwd", "attn_bwd", "gemm", "moe", "dequant", "moe_decode",
                                                  "peer_sync", "decode_attn"])
    ap.add_argument("--seqlens", default="8192")
    ap.add_argument("--hq", type=int, default=64)
    ap.add_argument("--hkv", type=int, default=8)
    ap.add_argument("--window", type=int, default=0)
    ap.add_argument("--m", type=int, default=16384)
    ap.add_argument("--n", type=int, default=5760)
    ap.add_argument("--k", type=int, default=2880)
    ap.add_argument("--tokens", type=int, default=32768)
    ap.add_argument("--experts", type=int, default=128)
    ap.add_argument("--path", choices=["mxfp4", "dequant"], default="mxfp4")
    ap.add_argument("--iters", type=int, default=10)
    args = ap.parse_args()
    if args.op == "attn_fwd":
        r = bench_attention(args, False)
    elif args.op == "attn_bwd":
        r = bench_attention(args, True)
    elif args.op == "gemm":
        r = bench_gemm(args)
    elif args.op == "dequant":
        r = bench_dequant(args)
    elif args.op == "moe_decode":
        r = bench_moe_decode(args)
    elif args.op == "peer_sync":
        r = bench_peer_sync(args)
    elif args.op == "decode_attn":
        r = bench_decode_attn(args)
    else:
        r = bench_moe(args)
    peak_tf, peak_bw, kind = _peaks()
    if "bytes" in r:
        gbs = r["bytes"] / (r["ms"] / 1e3) / 1e9
        extra = {k: v for k, v in r.items() if k not in ("bytes", "ms")}
        print(json.dumps({"op": args.op, "ms": round(r["ms"], 4), "gb_per_s": round(gbs, 1),
                          f"frac_of_{kind}_hbm": round(gbs / peak_bw, 3), **extra,
                          "args": vars(args)}))
        return
    tf = r["flops"] / (r["ms"] / 1e3) / 1e12
    print(json.dumps({"op": args.op, "ms": round(r["ms"], 4), "tflops": round(tf, 1),
                      f"frac_of_{kind}_bf16_peak": round(tf / peak_tf, 3), "args": vars(args)}))


if __name__ == "__main__":
    main()
