"""Rollout throughput of the built-in engine: gpt-oss random-init weights with MXFP4 experts,
``--requests`` concurrent trajectories, each a ``--prompt``-token random prompt that generates
``--gen`` tokens at temperature 1.0, paged bf16 KV cache, continuous batching.  Under torchrun
the engine runs tensor-parallel over the launched ranks (one GPU each; attention heads and
experts split, partial sums reduced by the fused NVLink all-reduce + RMSNorm kernel).

    python -m agent_factory_3_b200.benchmarks.rollout_decode --model gpt-oss-120b --requests 128
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m agent_factory_3_b200.benchmarks.rollout_decode

Prints one JSON line: wall time, generated tokens/s over the whole run, and the decode-phase
rate (tokens/s from the moment every request has its first token until the last finishes),
plus the mean engine step time in the decode phase.
"""
from __future__ import annotations

import argparse
import json
import os
import threading
import time

import torch


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="gpt-oss-120b")
    ap.add_argument("--layers", type=int, default=None, help="(smoke only) override layer count")
    ap.add_argument("--requests", type=int, default=128)
    ap.add_argument("--prompt", type=int, default=2048)
    ap.add_argument("--gen", type=int, default=256)
    ap.add_argument("--page-size", type=int, default=64)
    ap.add_argument("--max-prefill-tokens", type=int, default=16384)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--spec", choices=["none", "block", "ngram"], default="none",
                    help="speculative decoding: block = 1-layer random-init block draft model")
    ap.add_argument("--spec-block", type=int, default=8)
    ap.add_argument("--cuda-graphs", action="store_true", help="replay decode steps from CUDA graphs (TP=1)")
    ap.add_argument("--trace", default=None,
                    help="write a per-kernel device-time table of the run to this path (profiled "
                         "run: its throughput is not a benchmark number)")
    a = ap.parse_args()

    from ..engine.scheduler import Engine, Request
    from ..models.gpt_oss import GptOssConfig, GptOssForCausalLM
    cfg = GptOssConfig.preset(a.model)
    if a.layers:
        cfg.num_hidden_layers = a.layers
        cfg.layer_types = cfg.layer_types[: a.layers]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
        cpu_group = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=600))
    dev = torch.device("cuda", torch.cuda.current_device())
    t0 = time.perf_counter()
    model = GptOssForCausalLM(cfg, device=dev).init_random(a.seed).eval()
    torch.cuda.synchronize()
    init_s = time.perf_counter() - t0
    pages_per_req = (a.prompt + a.gen + a.page_size - 1) // a.page_size + 1
    tp = shards = None
    if world > 1:
        from ..engine.tp import TPContext, broadcast_model, shard_model
        broadcast_model(model)
        shards = shard_model(model, rank, world, free_full=True)
        torch.cuda.empty_cache()
        tp = TPContext(None, cpu_group, dev, max_tokens=a.max_prefill_tokens + a.requests,
                       hidden=cfg.hidden_size)
    drafter = None
    if a.spec == "block":
        from ..engine.spec import BlockDraftModel
        drafter = BlockDraftModel.from_target(model, n_layers=1, block=a.spec_block, seed=a.seed + 1)
    elif a.spec == "ngram":
        from ..engine.spec import NgramDrafter
        drafter = NgramDrafter(block=a.spec_block)
    eng = Engine(model, num_pages=a.requests * pages_per_req + 64, page_size=a.page_size,
                 max_running=a.requests, max_prefill_tokens=a.max_prefill_tokens, tp=tp,
                 tp_shards=shards, drafter=drafter, cuda_graphs=a.cuda_graphs and world == 1)
    if rank != 0:
        eng.runner.follow()
        tp.shutdown()
        dist.destroy_process_group()
        return
    eng.start()
    g = torch.Generator().manual_seed(a.seed)
    lock = threading.Lock()
    state = {"first": 0, "done": 0, "t_all_first": None, "t_end": None}
    all_done = threading.Event()

    def make_cb(req):
        seen = {"first": False}

        def cb(out):
            with lock:
                if not seen["first"] and len(req.output_ids) > 0:
                    seen["first"] = True
                    state["first"] += 1
                    if state["first"] == a.requests:
                        state["t_all_first"] = time.perf_counter()
                if out["finished"]:
                    state["done"] += 1
                    if state["done"] == a.requests:
                        state["t_end"] = time.perf_counter()
                        all_done.set()
        return cb

    # warm-up: one short request compiles nothing but touches every kernel once
    warm = Request(input_ids=torch.randint(0, cfg.vocab_size, (64,), generator=g).tolist(),
                   max_new_tokens=4, temperature=1.0, seed=1)
    ev = threading.Event()
    warm.on_output = lambda out: ev.set() if out["finished"] else None
    eng.submit(warm)
    ev.wait(600)
    steps0 = eng.step_count
    reqs = []
    for i in range(a.requests):
        r = Request(input_ids=torch.randint(0, cfg.vocab_size, (a.prompt,), generator=g).tolist(),
                    max_new_tokens=a.gen, temperature=1.0, seed=i, stop_token_ids=[],
                    stream=True)   # per-step callbacks: the first token of each request is seen
        r.on_output = make_cb(r)
        reqs.append(r)
    prof = None
    if a.trace:
        from torch.profiler import ProfilerActivity, profile
        prof = profile(activities=[ProfilerActivity.CUDA])
        prof.__enter__()
    t_start = time.perf_counter()
    for r in reqs:
        eng.submit(r)
    ok = all_done.wait(3600)
    if prof is not None:
        torch.cuda.synchronize()
        prof.__exit__(None, None, None)
        with open(a.trace, "w") as f:
            f.write(prof.key_averages().table(sort_by="cuda_time_total", row_limit=40))
    steps = eng.step_count - steps0
    eng.stop()
    gen = sum(len(r.output_ids) for r in reqs)
    wall = (state["t_end"] or time.perf_counter()) - t_start
    err = None
    try:
        from ..ops._ext import check_device_error
        check_device_error()
    except Exception as e:  # noqa: BLE001
        err = str(e)[:200]
    out = {"metric": "rollout generated tokens/s", "tp": world, "model": a.model,
           "layers": cfg.num_hidden_layers, "requests": a.requests, "prompt": a.prompt,
           "gen": a.gen, "completed": ok, "generated_tokens": gen, "wall_s": round(wall, 2),
           "gen_tok_per_s": round(gen / wall, 1), "engine_steps": steps, "init_s": round(init_s, 1)}
    if state["t_all_first"] and state["t_end"]:
        dec = state["t_end"] - state["t_all_first"]
        out["decode_phase_s"] = round(dec, 2)
        out["decode_tok_per_s"] = round((gen - a.requests) / dec, 1) if dec > 0 else None
        out["decode_step_ms"] = round(dec / max(1, a.gen - 1) * 1000, 2)
    if tp is not None:
        out["fused_allreduce_calls"] = tp.fused_calls
    if eng.runner.graphs is not None:
        out["cuda_graphs"] = {"captured": len(eng.runner.graphs.graphs),
                              "replays": eng.runner.graphs.replays}
    if drafter is not None:
        out["spec"] = {"drafter": a.spec, "block": a.spec_block,
                       "accept_length": round(eng.spec_accept_length, 3),
                       "verifies": eng.spec_verifies}
    if err:
        out["device_error"] = err
    print(json.dumps(out), flush=True)
    if world > 1:
        tp.shutdown()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
