"""Rollout throughput of the built-in engine on one GPU (one-GPU slice):
gpt-oss random-init weights with MXFP4 experts, ``--requests`` concurrent trajectories, each a
``--prompt``-token random prompt that generates ``--gen`` tokens at temperature 1.0, paged bf16
KV cache, continuous batching.

    python -m agent_factory_3_b200.benchmarks.rollout_decode --model gpt-oss-120b --requests 128

Prints one JSON line: wall time, generated tokens/s over the whole run, and the decode-phase
rate (tokens/s from the moment every request has its first token until the last finishes),
plus the mean engine step time in the decode phase.
"""
from __future__ import annotations

import argparse
import json
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
    a = ap.parse_args()

    from ..engine.scheduler import Engine, Request
    from ..models.gpt_oss import GptOssConfig, GptOssForCausalLM
    cfg = GptOssConfig.preset(a.model)
    if a.layers:
        cfg.num_hidden_layers = a.layers
        cfg.layer_types = cfg.layer_types[: a.layers]
    dev = torch.device("cuda")
    t0 = time.perf_counter()
    model = GptOssForCausalLM(cfg, device=dev).init_random(a.seed).eval()
    torch.cuda.synchronize()
    init_s = time.perf_counter() - t0
    pages_per_req = (a.prompt + a.gen + a.page_size - 1) // a.page_size + 1
    eng = Engine(model, num_pages=a.requests * pages_per_req + 64, page_size=a.page_size,
                 max_running=a.requests, max_prefill_tokens=a.max_prefill_tokens).start()
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
                    max_new_tokens=a.gen, temperature=1.0, seed=i, stop_token_ids=[])
        r.on_output = make_cb(r)
        reqs.append(r)
    t_start = time.perf_counter()
    for r in reqs:
        eng.submit(r)
    ok = all_done.wait(3600)
    steps = eng.step_count - steps0
    eng.stop()
    gen = sum(len(r.output_ids) for r in reqs)
    wall = (state["t_end"] or time.perf_counter()) - t_start
    out = {"metric": "rollout generated tokens/s (one GPU)", "model": a.model,
           "layers": cfg.num_hidden_layers, "requests": a.requests, "prompt": a.prompt,
           "gen": a.gen, "completed": ok, "generated_tokens": gen, "wall_s": round(wall, 2),
           "gen_tok_per_s": round(gen / wall, 1), "engine_steps": steps, "init_s": round(init_s, 1)}
    if state["t_all_first"] and state["t_end"]:
        dec = state["t_end"] - state["t_all_first"]
        out["decode_phase_s"] = round(dec, 2)
        out["decode_tok_per_s"] = round((gen - a.requests) / dec, 1) if dec > 0 else None
        out["decode_step_ms"] = round(dec / max(1, a.gen - 1) * 1000, 2)
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
