"""Collective benchmarks on one NVLink box, one rank per GPU (run under torchrun):

  * ``allreduce``: the engine's fused tensor-parallel reduction (partials in IPC-mapped
    buffers -> one kernel: NVLink all-reduce + residual add + RMSNorm) against the NCCL
    baseline doing the same work (``all_reduce`` of the partial, then residual add + RMSNorm);
  * ``weight_sync``: the fused fp32 -> bf16 cast + NVLink store of trainer tensors (rank 1) into
    rank 0's staging buffer against NCCL ``send``/``recv`` of the same bf16 bytes after a
    separate cast;
  * ``grad_rs``: the trainer's pushed gradient reduce-scatter against NCCL reduce-scatter;
  * ``expert_gather``: the fused NVLink gather + MXFP4 dequantisation of sharded experts
    against NCCL all-gather + dequantisation.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m agent_factory_3_b200.benchmarks.collectives --op allreduce

Device time per call with CUDA events on each rank, reported as the max over ranks, plus the
NVLink roofline of the fused path: the time the bytes that must cross NVLink need at the
measured 770 GB/s per direction per GPU.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist

LINK_GBS = 770.0     # measured peer copy, GB/s per direction per GPU


def _max_over_ranks(v: float) -> float:
    t = torch.tensor([v], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _time(fn, iters, warmup=5):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def bench_allreduce(a, rank, world, dev):
    from ..engine.tp import TPContext
    from ..ops._ext import check_device_error
    from ..ops.norm import rmsnorm
    H = a.hidden
    ctx = TPContext(None, None, dev, max_tokens=max(a.tokens), hidden=H, timeout_s=10.0)
    g = torch.Generator(device=dev).manual_seed(rank)
    w = torch.rand(H, generator=g, device=dev) + 0.5
    rows = []
    for T in a.tokens:
        res = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
        src = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)

        def fused():
            part = ctx.partial_buffer(T, H)
            part.copy_(src)                       # stands in for the GEMM writing its output
            ctx.allreduce_norm(part, res, w, 1e-5)

        def copy_only():
            ctx.partial_buffer(T, H).copy_(src)

        def nccl():
            part = src.clone()
            dist.all_reduce(part)
            x = (part.float() + res.float()).to(torch.bfloat16)
            rmsnorm(x, w, 1e-5)

        t_fused = _max_over_ranks(_time(fused, a.iters))
        t_copy = _max_over_ranks(_time(copy_only, a.iters))
        t_nccl = _max_over_ranks(_time(nccl, a.iters))
        nbytes = T * H * 2
        # one-shot: every rank reads the other ranks' partials once
        roof_ms = (world - 1) * nbytes / (LINK_GBS * 1e9) * 1e3
        rows.append({"tokens": T, "bytes": nbytes, "fused_ms": round(t_fused - t_copy, 4),
                     "fused_incl_copy_ms": round(t_fused, 4), "nccl_ar_add_norm_ms": round(t_nccl, 4),
                     "speedup_vs_nccl": round(t_nccl / max(1e-9, t_fused - t_copy), 2),
                     "nvlink_roofline_ms": round(roof_ms, 4),
                     "frac_of_roofline": round(roof_ms / max(1e-9, t_fused - t_copy), 3)})
    check_device_error()
    ctx.shutdown()
    return rows


def bench_weight_sync(a, rank, world, dev):
    from ..parallel.weight_sync import PeerWriter, StagingBuffer
    from ..ops._ext import check_device_error
    rows = []
    for mb in a.sizes_mb:
        n = int(mb * 1e6 / 2) // 8 * 8              # bf16 elements landing on rank 0
        shapes = {"w": (n,)}
        stage = StagingBuffer.for_tensors(shapes, dev) if rank == 0 else None
        handle = [stage.export() if rank == 0 else None]
        dist.broadcast_object_list(handle, src=0)
        src = torch.randn(n, device=dev)             # fp32 master copy
        writer = PeerWriter(handle[0], dev) if rank == 1 else None
        recv = torch.empty(n, device=dev, dtype=torch.bfloat16)

        def fused():
            if rank == 1:
                writer.write({"w": src}, stream_sync=False)

        def nccl():
            if rank == 1:
                dist.send(src.to(torch.bfloat16), dst=0)
            elif rank == 0:
                dist.recv(recv, src=1)

        t_fused = _max_over_ranks(_time(fused, a.iters))
        t_nccl = _max_over_ranks(_time(nccl, a.iters))
        nbytes = n * 2
        roof = nbytes / (LINK_GBS * 1e9) * 1e3
        rows.append({"bytes": nbytes, "fused_ms": round(t_fused, 4), "nccl_ms": round(t_nccl, 4),
                     "fused_gbs": round(nbytes / t_fused / 1e6, 1),
                     "nccl_gbs": round(nbytes / t_nccl / 1e6, 1),
                     "frac_of_roofline": round(roof / t_fused, 3)})
        dist.barrier()
        if writer is not None:
            writer.close()
        dist.barrier()
        del writer, stage
    check_device_error()
    return rows


def bench_grad_rs(a, rank, world, dev):
    """Data-parallel gradient reduce-scatter: the trainer's push path (every rank copies each
    owner's slice into the owner's IPC inbox with the copy engines, then one kernel waits for
    all ranks and sums the slots in rank order, with the sum of squares) against NCCL
    ``reduce_scatter_tensor`` of the same fp32 buffer.  Here the pushes are not overlapped with
    a backward pass (the trainer issues them during it), so this is the exposed worst case."""
    from ..ops._ext import check_device_error
    from ..parallel.grad_push import GradientPusher
    rows = []
    for mb in a.sizes_mb:
        S = int(mb * 1e6 / 4 / world) // 64 * 64           # fp32 elements per rank's slice
        flat = torch.randn(world * S, device=dev)
        shard = torch.empty(S, device=dev)
        dummy = torch.zeros(1, device=dev, requires_grad=True)
        pusher = GradientPusher([dummy], [0], flat, shard, timeout_s=60.0)
        pusher.ranges = [(0, world * S)]                   # the whole buffer is one tensor
        pusher.pushed = [False]
        ref = torch.empty(S, device=dev)

        def push():
            pusher.finish()

        def nccl():
            dist.reduce_scatter_tensor(ref, flat)

        t_push = _max_over_ranks(_time(push, a.iters))
        t_nccl = _max_over_ranks(_time(nccl, a.iters))
        torch.cuda.synchronize()
        err = (shard - ref).abs().max().item()
        nbytes = world * S * 4
        # every rank sends (W-1)/W of its buffer and receives as much
        roof = (world - 1) * S * 4 / (LINK_GBS * 1e9) * 1e3
        rows.append({"bytes": nbytes, "push_ms": round(t_push, 4), "nccl_rs_ms": round(t_nccl, 4),
                     "speedup_vs_nccl": round(t_nccl / t_push, 2),
                     "nvlink_roofline_ms": round(roof, 4), "push_frac_of_roofline": round(roof / t_push, 3),
                     "nccl_frac_of_roofline": round(roof / t_nccl, 3), "max_abs_diff_vs_nccl": err})
        pusher.check()
        pusher.close()
        dist.barrier()
    check_device_error()
    return rows


def bench_expert_gather(a, rank, world, dev):
    """Sharded frozen experts: one gpt-oss-120b layer's gate_up experts (128 x 5760 x 2880
    MXFP4) rebuilt as bf16 on every rank.  Fused: ``mxfp4_dequant_gather`` reads every owner's
    packed bytes and scales over NVLink and writes bf16 locally.  Baseline: NCCL all-gather of
    the packed bytes and scales, then the local dequantisation kernel."""
    from ..ops import mxfp4
    from ..ops._ext import check_device_error, ext
    from ..parallel.symm import PeerMappedBuffer
    E, N, K = 128, 5760, 2880
    epr = E // world
    nb, ns = epr * N * (K // 32) * 16, epr * N * (K // 32)
    off_s = (nb + 255) // 256 * 256
    buf = PeerMappedBuffer(off_s + ns, None, dev)
    g = torch.Generator(device=dev).manual_seed(rank)
    blocks_l = buf.local[:nb].view(epr, N, K // 32, 16)
    scales_l = buf.local[off_s:off_s + ns].view(epr, N, K // 32)
    blocks_l.copy_(torch.randint(0, 256, blocks_l.shape, generator=g, device=dev, dtype=torch.uint8))
    scales_l.copy_(torch.randint(118, 128, scales_l.shape, generator=g, device=dev, dtype=torch.uint8))
    torch.cuda.synchronize()
    dist.barrier()
    tabs = (torch.tensor(list(buf.bases), dtype=torch.int64, device=dev),
            torch.tensor([b + off_s for b in buf.bases], dtype=torch.int64, device=dev))
    out = torch.empty(E, N, K, device=dev, dtype=torch.bfloat16)
    full_b = torch.empty(E, N, K // 32, 16, device=dev, dtype=torch.uint8)
    full_s = torch.empty(E, N, K // 32, device=dev, dtype=torch.uint8)

    def fused():
        ext().mxfp4_dequant_gather(tabs[0], tabs[1], epr, out)

    def nccl():
        dist.all_gather_into_tensor(full_b, blocks_l)
        dist.all_gather_into_tensor(full_s, scales_l)
        mxfp4.dequantize(full_b, full_s, out=out)

    t_fused = _max_over_ranks(_time(fused, a.iters))
    t_nccl = _max_over_ranks(_time(nccl, a.iters))
    packed = E * N * K // 2 + E * N * K // 32
    link_ms = (world - 1) / world * packed / (LINK_GBS * 1e9) * 1e3
    hbm_ms = (E * N * K * 2 + packed / world) / 6541.5e9 * 1e3
    roof = max(link_ms, hbm_ms)
    row = {"layer_packed_bytes": packed, "fused_ms": round(t_fused, 4),
           "nccl_ag_dequant_ms": round(t_nccl, 4), "speedup_vs_nccl": round(t_nccl / t_fused, 2),
           "roofline_ms": round(roof, 4), "roofline_bound": "nvlink" if link_ms > hbm_ms else "hbm",
           "frac_of_roofline": round(roof / t_fused, 3)}
    check_device_error()
    dist.barrier()
    buf.close()
    return [row]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--op", choices=["allreduce", "weight_sync", "grad_rs", "expert_gather"],
                    default="allreduce")
    ap.add_argument("--tokens", type=int, nargs="+", default=[1, 8, 32, 128, 512, 2048, 8192])
    ap.add_argument("--hidden", type=int, default=2880)
    ap.add_argument("--sizes-mb", type=float, nargs="+", default=[1, 16, 64, 256, 1024])
    ap.add_argument("--iters", type=int, default=20)
    a = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dev = torch.device("cuda", torch.cuda.current_device())
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    try:
        rows = {"allreduce": bench_allreduce, "weight_sync": bench_weight_sync,
                "grad_rs": bench_grad_rs, "expert_gather": bench_expert_gather}[a.op](
                    a, rank, world, dev)
        if rank == 0:
            for r in rows:
                print(json.dumps({"op": a.op, "world": world, **r}), flush=True)
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
