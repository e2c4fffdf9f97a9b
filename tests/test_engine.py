"""Rollout engine on the tiny model (CPU reference kernels; the same code drives the sm_100a
kernels on GPU): greedy decoding equals a full recompute, prefix caching, routed experts,
pause/abort/continue, LoRA hot-swap and merged-weight reload through the HTTP API."""
import asyncio
import base64

import numpy as np
import pytest
import torch
from aiohttp.test_utils import TestClient, TestServer

from agent_factory_3_b200.engine.kv_cache import PagedKVCache
from agent_factory_3_b200.engine.scheduler import Engine
from agent_factory_3_b200.engine.server import build_app
from agent_factory_3_b200.models.gpt_oss import GptOssConfig, GptOssForCausalLM, LoraConfig


def tiny_model(dev="cpu", lora=None, dtype=torch.float32):
    cfg = GptOssConfig.tiny()
    m = GptOssForCausalLM(cfg, lora=lora, device=dev, dtype=dtype).init_random(0)
    m.eval()
    return m


def assert_greedy(model, prompt, out, tol=1e-4):
    """Each greedy token must be a (near-)argmax of a full recompute over prompt + out: the
    engine thread's CPU reductions run in another order, and random-init models have
    near-tied logits, so token sequences alone are a brittle comparison."""
    ids = list(prompt) + list(out[:-1])
    with torch.no_grad():
        h = model.forward_hidden(torch.tensor(ids), torch.arange(len(ids)),
                                 torch.tensor([0, len(ids)], dtype=torch.int32))
        lg = model.logits(h[len(prompt) - 1:]).float()
    chosen = lg[torch.arange(len(out)), torch.tensor(out)]
    assert bool((chosen >= lg.max(-1).values - tol).all()), (out, lg.argmax(-1).tolist())


def test_kv_cache_prefix_and_eviction():
    kv = PagedKVCache(2, 6, 4, 2, 16, 2, "cpu", torch.float32)
    toks = list(range(12))
    pages, _ = kv.match_prefix(toks, "s")
    assert pages == []
    p = kv.allocate(3)
    prev = b""
    for i, pg in enumerate(p):
        prev = kv.chain(prev, toks[i * 4:(i + 1) * 4], "s")
        kv.register(pg, prev)
    kv.release(p)
    got, _ = kv.match_prefix(toks + [99], "s")
    assert got == p
    assert kv.match_prefix(toks, "other-salt")[0] == []
    kv.release(got)
    kv.allocate(6)   # evicts the cached pages
    assert kv.match_prefix(toks, "s")[0] == []


async def _client(engine):
    client = TestClient(TestServer(build_app(engine)))
    await client.start_server()
    return client


def test_engine_greedy_matches_recompute_and_routing():
    model = tiny_model()
    eng = Engine(model, num_pages=64, page_size=16, max_prefill_tokens=64).start()
    prompt = list(range(5, 45))

    async def run():
        c = await _client(eng)
        try:
            body = {"input_ids": prompt, "sampling_params": {"max_new_tokens": 6, "temperature": 0.0},
                    "return_logprob": True, "return_routed_experts": True, "return_entropy": True}
            r = await (await c.post("/generate", json=body)).json()
            r2 = await (await c.post("/generate", json=body)).json()
            loads = await (await c.get("/v1/loads")).json()
            return r, r2, loads
        finally:
            await c.close()

    try:
        r, r2, loads = asyncio.run(run())
    finally:
        eng.stop()
    assert len(r["output_ids"]) == 6
    assert_greedy(model, prompt, r["output_ids"])
    meta = r["meta_info"]
    assert meta["finish_reason"]["type"] == "length" and meta["completion_tokens"] == 6
    assert len(meta["output_token_logprobs"]) == 6 and len(meta["output_token_entropy"]) == 6
    rt = np.frombuffer(base64.b64decode(meta["routed_experts"]), dtype=np.int32)
    assert rt.size == (len(prompt) + 6 - 1) * 2 * 2
    # the second identical request hits the prefix cache and decodes the same tokens
    assert r2["output_ids"] == r["output_ids"] and r2["meta_info"]["cached_tokens"] >= 32
    rt2 = np.frombuffer(base64.b64decode(r2["meta_info"]["routed_experts"]), dtype=np.int32)
    assert np.array_equal(rt, rt2)
    assert "num_running_reqs" in loads["loads"][0]


def test_pause_abort_continue_and_weight_version():
    model = tiny_model()
    eng = Engine(model, num_pages=64, page_size=16).start()

    async def run():
        c = await _client(eng)
        try:
            body = {"input_ids": list(range(10, 30)),
                    "sampling_params": {"max_new_tokens": 400, "temperature": 1.0}}
            task = asyncio.create_task((await c.post("/generate", json=body)).json()) if False else None
            fut = asyncio.ensure_future(c.post("/generate", json=body))
            await asyncio.sleep(0.3)
            await c.post("/pause_generation", json={"mode": "abort"})
            r = await (await fut).json()
            # a request sent while paused waits for continue
            await c.post("/update_weight_version", json={"new_version": "7"})
            fut2 = asyncio.ensure_future(c.post("/generate", json={
                "input_ids": [1, 2, 3], "sampling_params": {"max_new_tokens": 2}}))
            await asyncio.sleep(0.2)
            assert not fut2.done()
            await c.post("/continue_generation", json={})
            r2 = await (await fut2).json()
            return r, r2
        finally:
            await c.close()

    try:
        r, r2 = asyncio.run(run())
    finally:
        eng.stop()
    assert r["meta_info"]["finish_reason"]["type"] == "abort"
    assert len(r["output_ids"]) < 400
    assert r2["meta_info"]["weight_version"] == "7"


def test_lora_hot_swap_and_merged_reload(tmp_path):
    from agent_factory_3_b200.trainer.model_trainer import ModelTrainer
    from agent_factory_3_b200.trainer.training_config import TrainingConfig
    lora = LoraConfig(r=4, lora_alpha=8, target_modules=["q_proj", "v_proj", "o_proj"])
    tcfg = TrainingConfig(model_id="tiny", lora_r=4, lora_alpha=8,
                          lora_target_modules=["q_proj", "v_proj", "o_proj"], random_init_seed=0)
    tr = ModelTrainer(tcfg, device="cpu")
    with torch.no_grad():
        for p in tr.model.parameters():
            if p.requires_grad:
                p.normal_(0, 0.3)
    tr.save_model(str(tmp_path / "adapter"))
    tr.save_merged_weights(str(tmp_path / "merged"))
    served = GptOssForCausalLM(GptOssConfig.tiny(), lora=lora, dtype=torch.float32)
    served.load_state_dict({k: v for k, v in tr.model.state_dict().items() if "lora" not in k}, strict=False)
    served.eval()
    eng = Engine(served, num_pages=64, page_size=16).start()
    prompt = list(range(3, 30))

    async def run():
        c = await _client(eng)
        try:
            body = {"input_ids": prompt, "sampling_params": {"max_new_tokens": 5, "temperature": 0.0}}
            base = await (await c.post("/generate", json=body)).json()
            r = await c.post("/load_lora_adapter", json={"lora_name": "policy",
                                                          "lora_path": str(tmp_path / "adapter")})
            assert r.status == 200
            adapted = await (await c.post("/generate", json=dict(body, lora_path="policy"))).json()
            await c.post("/update_weights_from_disk", json={"model_path": str(tmp_path / "merged"),
                                                            "flush_cache": True, "weight_version": "m1"})
            merged = await (await c.post("/generate", json=body)).json()
            bad = await c.post("/unload_lora_adapter", json={"lora_name": "missing"})
            return base, adapted, merged, bad.status
        finally:
            await c.close()

    try:
        base, adapted, merged, bad = asyncio.run(run())
    finally:
        eng.stop()
    assert_greedy(tr.model, prompt, adapted["output_ids"])
    assert_greedy(tr.model, prompt, merged["output_ids"])   # LoRA folded into the base weights
    assert merged["meta_info"]["weight_version"] == "m1"
    assert bad == 400


def test_top_logprobs_are_the_k_best_tokens():
    """``top_logprobs_num`` returns, per generated token, the k most likely tokens with their
    log-probabilities under the request's temperature, best first; under greedy decoding the
    first alternative is the generated token itself."""
    import threading

    from agent_factory_3_b200.engine.scheduler import Request
    model = tiny_model()
    eng = Engine(model, num_pages=64, page_size=16).start()
    try:
        prompt = list(range(5, 25))
        done = threading.Event()
        box = {}
        r = Request(input_ids=prompt, max_new_tokens=4, temperature=0.0, return_logprob=True,
                    top_logprobs_num=5)
        r.on_output = lambda out: (box.update(out), done.set()) if out["finished"] else None
        eng.submit(r)
        assert done.wait(120)
    finally:
        eng.stop()
    meta = box["meta_info"]
    out = box["output_ids"]
    tops = meta["output_top_logprobs"]
    assert len(tops) == len(out) == 4
    ids = prompt + out[:-1]
    with torch.no_grad():
        h = model.forward_hidden(torch.tensor(ids), torch.arange(len(ids)),
                                 torch.tensor([0, len(ids)], dtype=torch.int32))
        lp = torch.log_softmax(model.logits(h[len(prompt) - 1:]).float(), -1)
    for pos, row in enumerate(tops):
        assert len(row) == 5 and all(len(e) == 3 for e in row)
        vals = [e[0] for e in row]
        assert vals == sorted(vals, reverse=True)
        assert row[0][1] == out[pos]
        want_v, want_i = lp[pos].topk(5)
        assert [e[1] for e in row][:2] == want_i.tolist()[:2] or abs(vals[0] - vals[1]) < 1e-4
        assert abs(vals[0] - float(want_v[0])) < 1e-3


def _adapter_params(model, seed):
    g = torch.Generator().manual_seed(seed)
    return {k: torch.randn(p.shape, generator=g) * 0.2 for k, p in model.lora_param_dict().items()}


def test_mixed_adapter_step_matches_single_adapter_runs():
    """One step over sequences of adapter A, adapter B and no adapter (stacked-rank LoRA with
    per-row rank masks) gives each sequence the logits of a step run with only its adapter."""
    from agent_factory_3_b200.engine.model_runner import ModelRunner, StepItem
    lora = LoraConfig(r=4, lora_alpha=8, target_modules=["q_proj", "k_proj", "v_proj", "o_proj",
                                                         "gate_up_proj", "down_proj"])
    model = tiny_model(lora=lora)
    cfg = model.cfg
    bank = {"A": _adapter_params(model, 1), "B": _adapter_params(model, 2)}
    prompts = {"A": list(range(3, 40)), "B": list(range(50, 71)), None: list(range(80, 93))}

    def kv():
        return PagedKVCache(cfg.num_hidden_layers, 32, 16, cfg.num_key_value_heads, cfg.head_dim,
                            cfg.num_experts_per_tok, "cpu", torch.float32)
    pages = {"A": [0, 1, 2], "B": [3, 4], None: [5]}
    runner = ModelRunner(model, kv(), lora_active=True)
    items = [StepItem(prompts[a], 0, pages[a], adapter=a) for a in ("A", "B", None)]
    mixed = runner.forward_mixed(items, bank).logits
    params = model.lora_param_dict()
    for j, a in enumerate(("A", "B", None)):
        single = ModelRunner(model, kv(), lora_active=a is not None)
        if a is not None:
            with torch.no_grad():
                for k, p in params.items():
                    p.copy_(bank[a][k])
        ref = single.forward([StepItem(prompts[a], 0, pages[a])]).logits[0]
        torch.testing.assert_close(mixed[j], ref, rtol=1e-4, atol=1e-4)


def test_engine_batches_requests_of_different_adapters_together():
    lora = LoraConfig(r=4, lora_alpha=8, target_modules=["q_proj", "v_proj", "o_proj",
                                                         "gate_up_proj", "down_proj"])
    model = tiny_model(lora=lora)
    eng = Engine(model, num_pages=64, page_size=16)
    calls = {"mixed": 0}
    orig = eng.runner.forward_mixed

    def counting(items, bank):
        calls["mixed"] += 1
        return orig(items, bank)
    eng.runner.forward_mixed = counting
    eng.start()
    try:
        eng.control("apply_lora_params", "A", _adapter_params(model, 1))
        eng.control("apply_lora_params", "B", _adapter_params(model, 2))

        async def run():
            c = await _client(eng)
            try:
                bodies = [{"input_ids": list(range(3 + 7 * i, 20 + 7 * i)),
                           "sampling_params": {"max_new_tokens": 6, "temperature": 0.0},
                           **({"lora_path": a} if a else {})}
                          for i, a in enumerate(("A", "B", None, "A"))]
                res = await asyncio.gather(*(c.post("/generate", json=b) for b in bodies))
                outs = [await r.json() for r in res]
                bad = await c.post("/generate", json=dict(bodies[0], lora_path="missing"))
                return outs, (await bad.json())
            finally:
                await c.close()
        outs, bad = asyncio.run(run())
    finally:
        eng.stop()
    assert all(len(o["output_ids"]) == 6 for o in outs)
    assert calls["mixed"] > 0
    assert bad["meta_info"]["finish_reason"]["type"] == "abort"


def test_server_accepts_the_reference_launch_flags():
    """The sglang flag set of a reference launch script parses, maps onto this engine's options
    and leaves a note for each flag that has no effect here."""
    from agent_factory_3_b200.engine.server import build_arg_parser, resolve_args
    argv = ["--model-path", "/models/gpt-oss-120b", "--tp-size", "2", "--dtype", "bfloat16",
            "--attention-backend", "fa3", "--kv-cache-dtype", "fp8_e4m3",
            "--mem-fraction-static", "0.82", "--max-running-requests", "128",
            "--swa-full-tokens-ratio", "0.1", "--trust-remote-code", "--host", "0.0.0.0",
            "--port", "30000", "--scheduler-recv-interval", "16", "--log-level", "info",
            "--enable-return-routed-experts", "--weight-loader-disable-mmap",
            "--disable-cuda-graph-padding", "--enable-metrics", "--enable-cache-report",
            "--speculative-algorithm", "DFLASH", "--speculative-draft-model-path", "/models/d",
            "--speculative-draft-model-quantization", "fp8", "--speculative-dflash-block-size", "10"]
    a = build_arg_parser().parse_args(argv)
    notes = resolve_args(a, world=2)
    assert a.model == "/models/gpt-oss-120b" and a.tp_size == 2 and a.port == 30000
    assert a.speculative_algorithm == "block" and a.speculative_num_draft_tokens == 10
    assert a.mem_fraction_static == 0.82 and a.num_pages is None
    text = " ".join(notes)
    assert "stays bf16" in text and "--attention-backend" in text and "--enable-metrics" in text
    with pytest.raises(SystemExit):          # two ranks asked for, one process launched
        resolve_args(build_arg_parser().parse_args(["--tp-size", "2"]), world=1)
    with pytest.raises(SystemExit):
        resolve_args(build_arg_parser().parse_args(["--num-pages", "8", "--mem-fraction-static",
                                                    "0.5"]), world=1)


def test_kv_pages_for_memory_fraction():
    cfg = GptOssConfig.preset("gpt-oss-120b")
    page = PagedKVCache.bytes_per_page(cfg.num_hidden_layers, 64, cfg.num_key_value_heads,
                                       cfg.head_dim, cfg.num_experts_per_tok)
    assert page == 36 * 64 * (2 * 8 * 64 * 2 + 4)
    gib = 1 << 30
    n = PagedKVCache.pages_for_memory_fraction(0.82, 180 * gib, 70 * gib, page)
    assert n == int((0.82 * 180 * gib - 70 * gib) // page) and n > 0
    with pytest.raises(ValueError):
        PagedKVCache.pages_for_memory_fraction(0.3, 180 * gib, 70 * gib, page)
