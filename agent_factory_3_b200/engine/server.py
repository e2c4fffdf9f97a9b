"""sglang-compatible HTTP server of the rollout engine.

Endpoints (contract of the sglang API the reference drives, see rollout/llm_backend/
sglang_backend.py and trainer/sglang_controller.py of agent-factory-3):
  POST /generate                 input_ids, sampling_params, stream, return_logprob,
                                 logprob_start_len, return_entropy, top_logprobs_num,
                                 return_routed_experts, lora_path, extra_key
  POST /pause_generation         {"mode": "abort" | "in_place"}
  POST /continue_generation
  POST /load_lora_adapter        {"lora_name", "lora_path"}
  POST /unload_lora_adapter      {"lora_name"}
  POST /update_weight_version    {"new_version"}
  POST /flush_cache
  POST /update_weights_from_disk {"model_path", "flush_cache", "weight_version"}
  POST /lora_sync/export         CUDA IPC handle of a LoRA staging buffer (same machine)
  POST /lora_sync/apply          {"lora_name", "weight_version", "flush_cache"}: staged -> model
  GET  /v1/loads, /health, /get_model_info, /get_server_info
Control calls return once the engine thread has applied them, so a weight sync needs no
fixed sleeps (the reference sleeps >= 13 s per LoRA sync waiting for sglang's asynchronous
scheduler).

    python -m agent_factory_3_b200.engine.server --model gpt-oss-120b --port 30000
"""
from __future__ import annotations

import argparse
import asyncio
import json
import logging

from aiohttp import web

from .scheduler import Engine, Request

logger = logging.getLogger(__name__)


def _request_from_json(body: dict) -> Request:
    sp = body.get("sampling_params") or {}
    ids = body.get("input_ids")
    if not isinstance(ids, list) or not ids:
        raise web.HTTPBadRequest(text="input_ids must be a non-empty list of token ids")
    return Request(
        input_ids=[int(t) for t in ids], max_new_tokens=int(sp.get("max_new_tokens", 128)),
        temperature=float(sp.get("temperature", 1.0)), top_p=float(sp.get("top_p", 1.0)),
        top_k=int(sp.get("top_k", -1)), min_p=float(sp.get("min_p") or 0.0),
        seed=sp.get("sampling_seed"), stop_token_ids=[int(t) for t in sp.get("stop_token_ids") or []],
        return_logprob=bool(body.get("return_logprob", False)),
        return_entropy=bool(body.get("return_entropy", False)),
        top_logprobs_num=int(body.get("top_logprobs_num") or 0),
        return_routed_experts=bool(body.get("return_routed_experts", False)),
        lora_path=body.get("lora_path"), extra_key=body.get("extra_key"),
        stream=bool(body.get("stream", False)))


def build_app(engine: Engine, model_info: dict | None = None, faults=None) -> web.Application:
    """``faults``: an ``engine.faults.FaultPlan`` (default: from AF3_ENGINE_FAULTS) that makes
    /generate drop, delay or abort requests on purpose, for client robustness tests."""
    app = web.Application(client_max_size=1 << 30)
    if faults is None:
        from .faults import FaultPlan
        faults = FaultPlan.from_env()

    async def generate(request: web.Request):
        body = await request.json()
        req = _request_from_json(body)
        vocab = engine.model.cfg.vocab_size
        if min(req.input_ids) < 0 or max(req.input_ids) >= vocab:
            # never let an out-of-range id reach the embedding gather on the device
            return web.json_response({"error": f"input_ids must lie in [0, {vocab})"}, status=400)
        abort_at = None
        if faults is not None:
            if faults.delay_ms > 0:
                await asyncio.sleep(faults.delay_ms / 1000.0)
            if faults.should_drop():
                return web.json_response({"error": "injected fault: request dropped"}, status=503)
            abort_at = faults.abort_point()
            faults.aborted += int(abort_at is not None)
        req.abort_after_tokens = abort_at
        loop = asyncio.get_running_loop()
        q: asyncio.Queue = asyncio.Queue()
        req.on_output = lambda out: loop.call_soon_threadsafe(q.put_nowait, out)
        engine.submit(req)
        if not req.stream:
            try:
                while True:
                    out = await q.get()
                    if out["finished"]:
                        return web.json_response({"output_ids": out["output_ids"],
                                                  "meta_info": out["meta_info"]})
            except asyncio.CancelledError:      # client went away: free the request's pages
                engine.control("abort_request", req, wait=False)
                raise
        resp = web.StreamResponse(headers={"Content-Type": "text/event-stream",
                                           "Cache-Control": "no-cache"})
        await resp.prepare(request)
        try:
            while True:
                out = await q.get()
                chunk = {"output_ids": out["output_ids"], "meta_info": out["meta_info"]}
                await resp.write(f"data: {json.dumps(chunk)}\n\n".encode())
                if out["finished"]:
                    break
            await resp.write(b"data: [DONE]\n\n")
        except (ConnectionResetError, asyncio.CancelledError):
            # the client closed the stream (pause / stop / interrupt): abort the request so it
            # stops generating and releases its pages; its prefix stays cached for a re-issue
            engine.control("abort_request", req, wait=False)
        return resp

    def control(cmd, *args):
        return asyncio.get_running_loop().run_in_executor(None, lambda: engine.control(cmd, *args))

    async def pause(request):
        body = await request.json() if request.can_read_body else {}
        await control("pause", body.get("mode", "abort"))
        return web.json_response({"success": True})

    async def cont(request):
        await control("continue")
        return web.json_response({"success": True})

    async def load_lora(request):
        body = await request.json()
        try:
            await control("load_lora", body["lora_name"], body["lora_path"])
        except Exception as e:  # noqa: BLE001
            return web.json_response({"success": False, "message": str(e)}, status=400)
        return web.json_response({"success": True})

    async def unload_lora(request):
        body = await request.json()
        if body.get("lora_name") not in engine.loras:
            return web.json_response({"success": False,
                                      "message": f"LoRA adapter {body.get('lora_name')} does not exist"},
                                     status=400)
        await control("unload_lora", body["lora_name"])
        return web.json_response({"success": True})

    async def weight_version(request):
        body = await request.json()
        await control("update_weight_version", body.get("new_version"))
        return web.json_response({"success": True})

    async def flush(request):
        try:
            await control("flush_cache")
        except Exception as e:  # noqa: BLE001
            return web.json_response({"success": False, "message": str(e)}, status=400)
        return web.json_response({"success": True})

    async def update_weights(request):
        body = await request.json()
        await control("update_weights", body["model_path"], bool(body.get("flush_cache", True)))
        if body.get("weight_version") is not None:
            await control("update_weight_version", body["weight_version"])
        return web.json_response({"success": True, "message": "weights updated"})

    sync = {"stage": None}

    async def lora_sync_export(request):
        """CUDA IPC description of a staging buffer for the model's LoRA factors (same box)."""
        import base64

        from ..parallel.weight_sync import StagingBuffer
        if sync["stage"] is None:
            params = engine.model.lora_param_dict()
            if not params:
                return web.json_response({"success": False, "message": "model has no LoRA"}, status=400)
            dev = next(iter(params.values())).device
            sync["stage"] = StagingBuffer.for_tensors({k: tuple(v.shape) for k, v in params.items()}, dev)
        return web.json_response({"success": True,
                                  "handle": base64.b64encode(sync["stage"].export()).decode()})

    async def lora_sync_apply(request):
        body = await request.json() if request.can_read_body else {}
        if sync["stage"] is None:
            return web.json_response({"success": False, "message": "no staging buffer"}, status=400)
        await control("apply_lora_params", body.get("lora_name", "policy"), sync["stage"].tensors())
        if body.get("weight_version") is not None:
            await control("update_weight_version", body["weight_version"])
        if body.get("flush_cache", True):
            await control("flush_cache")
        return web.json_response({"success": True})

    async def loads(request):
        return web.json_response({"loads": [engine.loads()]})

    async def health(request):
        return web.Response(text="ok")

    async def info(request):
        return web.json_response(model_info or {"model": "gpt-oss"})

    app.router.add_post("/generate", generate)
    app.router.add_post("/pause_generation", pause)
    app.router.add_post("/continue_generation", cont)
    app.router.add_post("/load_lora_adapter", load_lora)
    app.router.add_post("/unload_lora_adapter", unload_lora)
    app.router.add_post("/update_weight_version", weight_version)
    app.router.add_post("/flush_cache", flush)
    app.router.add_post("/update_weights_from_disk", update_weights)
    app.router.add_post("/lora_sync/export", lora_sync_export)
    app.router.add_post("/lora_sync/apply", lora_sync_apply)
    app.router.add_get("/v1/loads", loads)
    app.router.add_get("/health", health)
    app.router.add_get("/get_model_info", info)
    app.router.add_get("/get_server_info", info)
    return app


# sglang launch flags that a reference launch script passes and that this engine accepts without
# acting on them (one attention path, one scheduler loop, no mmap'd loader, metrics always on)
_SGLANG_NO_EFFECT = ("--attention-backend", "--swa-full-tokens-ratio", "--scheduler-recv-interval",
                     "--log-level", "--speculative-draft-model-quantization")
_SGLANG_NO_EFFECT_SWITCHES = ("--trust-remote-code", "--weight-loader-disable-mmap",
                              "--disable-cuda-graph-padding", "--enable-metrics",
                              "--enable-cache-report", "--enable-return-routed-experts")


def build_arg_parser() -> argparse.ArgumentParser:
    """Engine flags, plus the sglang flags of the reference's launch scripts
    (examples/wordle/serve.sh:55-86): ``--model-path``, ``--tp-size``, ``--dtype``,
    ``--kv-cache-dtype``, ``--mem-fraction-static``, ``--speculative-algorithm DFLASH`` with
    ``--speculative-dflash-block-size`` and ``--speculative-draft-model-path``, and switches that
    need no action here (routed experts are returned whenever a request asks for them)."""
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", "--model-path", dest="model", default="gpt-oss-120b",
                    help="preset name or checkpoint directory")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=30000)
    ap.add_argument("--num-pages", type=int, default=None,
                    help="KV pages (default 8192, or sized by --mem-fraction-static)")
    ap.add_argument("--mem-fraction-static", type=float, default=None,
                    help="size the KV pool so this process uses this fraction of device memory")
    ap.add_argument("--page-size", type=int, default=64)
    ap.add_argument("--max-running-requests", type=int, default=128)
    ap.add_argument("--max-prefill-tokens", type=int, default=16384)
    ap.add_argument("--lora-r", "--max-lora-rank", dest="lora_r", type=int, default=0,
                    help="LoRA capacity (0 = no LoRA serving)")
    ap.add_argument("--lora-targets", "--lora-target-modules", dest="lora_targets",
                    default="q_proj,k_proj,v_proj,o_proj")
    ap.add_argument("--seed", "--random-seed", dest="seed", type=int, default=0)
    ap.add_argument("--tp-size", "--tp", dest="tp_size", type=int, default=None,
                    help="tensor-parallel ranks; must match the torchrun world (one process per GPU)")
    ap.add_argument("--dtype", default="bfloat16", choices=["auto", "bfloat16", "bf16"])
    ap.add_argument("--kv-cache-dtype", default="auto",
                    choices=["auto", "bfloat16", "bf16", "fp8_e4m3", "fp8_e5m2"],
                    help="the KV cache is bf16; fp8 requests are accepted and noted")
    ap.add_argument("--speculative-algorithm", type=str.lower, default="none",
                    choices=["none", "block", "ngram", "dflash"],
                    help="block (alias dflash): one-forward block draft model sharing the "
                         "target's embeddings")
    ap.add_argument("--speculative-num-draft-tokens", "--speculative-dflash-block-size",
                    dest="speculative_num_draft_tokens", type=int, default=8)
    ap.add_argument("--speculative-draft-layers", type=int, default=1)
    ap.add_argument("--speculative-draft-model-path", default=None,
                    help="accepted; the block draft is built from the target (its own layers "
                         "random-initialised from --seed)")
    ap.add_argument("--cuda-graphs", action="store_true", help="replay decode steps from CUDA graphs (TP=1)")
    for f in _SGLANG_NO_EFFECT:
        ap.add_argument(f, default=None, help=argparse.SUPPRESS)
    for f in _SGLANG_NO_EFFECT_SWITCHES:
        ap.add_argument(f, action="store_true", help=argparse.SUPPRESS)
    return ap


def resolve_args(a: argparse.Namespace, world: int) -> list[str]:
    """Checks and maps the compatibility flags in place; returns notes for the log."""
    notes = []
    if a.tp_size is not None and a.tp_size != world:
        raise SystemExit(f"--tp-size {a.tp_size} but {world} process(es): launch one process per "
                         f"GPU, e.g. torchrun --nproc-per-node {a.tp_size} -m "
                         "agent_factory_3_b200.engine.server ...")
    if a.speculative_algorithm == "dflash":
        a.speculative_algorithm = "block"
        notes.append(f"DFLASH -> block draft of {a.speculative_num_draft_tokens} tokens")
    if a.kv_cache_dtype.startswith("fp8"):
        notes.append(f"--kv-cache-dtype {a.kv_cache_dtype}: the KV cache stays bf16")
    if a.speculative_draft_model_path:
        notes.append("--speculative-draft-model-path: the block draft is built from the target")
    if a.num_pages is not None and a.mem_fraction_static is not None:
        raise SystemExit("give --num-pages or --mem-fraction-static, not both")
    ignored = [f for f in _SGLANG_NO_EFFECT if getattr(a, f[2:].replace("-", "_")) is not None]
    ignored += [f for f in _SGLANG_NO_EFFECT_SWITCHES if getattr(a, f[2:].replace("-", "_"))]
    if ignored:
        notes.append("accepted with no effect: " + " ".join(ignored))
    return notes


def main():
    import torch

    from ..models.gpt_oss import GptOssConfig, GptOssForCausalLM, LoraConfig
    from ..models.gpt_oss.checkpoint import load_checkpoint
    ap = build_arg_parser()
    a = ap.parse_args()
    from pathlib import Path
    import os
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    for note in resolve_args(a, world):
        if rank == 0:
            print(f"[engine] {note}", flush=True)
    p = Path(a.model)
    cfg = GptOssConfig.load(p / "config.json") if (p / "config.json").exists() else GptOssConfig.preset(a.model)
    lora = LoraConfig(r=a.lora_r, lora_alpha=2 * a.lora_r, target_modules=a.lora_targets.split(",")) if a.lora_r else None
    if world > 1:   # tensor parallel under torchrun: rank 0 serves HTTP, the others follow
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
        cpu_group = dist.new_group(backend="gloo", timeout=datetime.timedelta(days=1))
    dev = torch.device("cuda", torch.cuda.current_device())
    model = GptOssForCausalLM(cfg, lora=lora, device=dev)
    if p.is_dir():
        load_checkpoint(p, model)
    else:
        model.init_random(a.seed)
    model.eval()
    tp = shards = None
    if world > 1:
        from .tp import TPContext, broadcast_model, shard_model
        broadcast_model(model)
        shards = shard_model(model, rank, world, free_full=True)
        torch.cuda.empty_cache()
        tp = TPContext(None, cpu_group, dev, max_tokens=a.max_prefill_tokens + a.max_running_requests,
                       hidden=cfg.hidden_size)
    drafter = None
    if a.speculative_algorithm == "block":
        from .spec import BlockDraftModel
        drafter = BlockDraftModel.from_target(model, n_layers=a.speculative_draft_layers,
                                              block=a.speculative_num_draft_tokens, seed=a.seed + 1)
    elif a.speculative_algorithm == "ngram":
        from .spec import NgramDrafter
        drafter = NgramDrafter(block=a.speculative_num_draft_tokens)
    num_pages = a.num_pages if a.num_pages is not None else 8192
    if a.mem_fraction_static is not None:
        from .kv_cache import PagedKVCache
        free, total = torch.cuda.mem_get_info(dev)
        page_bytes = PagedKVCache.bytes_per_page(cfg.num_hidden_layers, a.page_size,
                                                 cfg.num_key_value_heads // world, cfg.head_dim,
                                                 cfg.num_experts_per_tok)
        num_pages = PagedKVCache.pages_for_memory_fraction(a.mem_fraction_static, total,
                                                           total - free, page_bytes)
        if rank == 0:
            print(f"[engine] --mem-fraction-static {a.mem_fraction_static:g}: {num_pages} KV pages "
                  f"of {a.page_size} tokens", flush=True)
    eng = Engine(model, num_pages=num_pages, page_size=a.page_size,
                 max_running=a.max_running_requests, max_prefill_tokens=a.max_prefill_tokens,
                 tp=tp, tp_shards=shards, drafter=drafter,
                 cuda_graphs=a.cuda_graphs and world == 1)
    if rank != 0:
        eng.runner.follow()
        tp.shutdown()
        return
    eng.start()
    try:
        web.run_app(build_app(eng, {"model": a.model, "num_hidden_layers": cfg.num_hidden_layers,
                                    "num_experts_per_tok": cfg.num_experts_per_tok}),
                    host=a.host, port=a.port)
    finally:
        eng.stop()
        if tp is not None:
            tp.shutdown()
    torch.cuda.synchronize()


if __name__ == "__main__":
    main()
