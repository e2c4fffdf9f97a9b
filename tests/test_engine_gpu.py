"""Rollout-engine kernels on B200 against PyTorch references: paged decode attention (sinks,
sliding window, GQA), KV page store/gather, Gumbel-max sampling statistics, and greedy engine
decoding equal to a full recompute on the GPU model."""
import asyncio
import base64
import math

import numpy as np
import pytest
import torch

from agent_factory_3_b200.ops import decode as D

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("window", [0, 48])
def test_decode_attention(dev, window):
    torch.manual_seed(0)
    B, hq, hkv, d, P, pages = 5, 16, 2, 64, 16, 64
    kp = torch.randn(pages, P, hkv, d, device=dev).bfloat16()
    vp = torch.randn(pages, P, hkv, d, device=dev).bfloat16()
    lens = torch.tensor([1, 17, 100, 300, 513], dtype=torch.int32)
    perm = torch.randperm(pages)
    pt = torch.zeros(B, 40, dtype=torch.int32)
    k = 0
    for b in range(B):
        n = (int(lens[b]) + P - 1) // P
        pt[b, :n] = perm[k:k + n]
        k += n
    q = torch.randn(B, hq * d, device=dev).bfloat16()
    sinks = torch.randn(hq, device=dev)
    out = D.decode_attention(q, kp, vp, pt.to(dev), lens.to(dev), sinks, hq, hkv, window)
    ref = D.decode_attention_reference(q.cpu().reshape(B, hq, d), kp.cpu(), vp.cpu(), pt, lens,
                                       sinks.cpu(), hq, hkv, window)
    torch.testing.assert_close(out.cpu().float(), ref, rtol=2e-2, atol=2e-2)


def test_kv_store_gather(dev):
    torch.manual_seed(1)
    kp = torch.zeros(8, 16, 2, 64, device=dev).bfloat16()
    vp = torch.zeros_like(kp)
    qkv = torch.randn(10, (4 + 4) * 64, device=dev).bfloat16()
    slots = torch.randperm(128)[:10].to(torch.int32).to(dev)
    D.kv_store(qkv, 256, 384, slots, kp, vp)
    back = torch.zeros_like(qkv)
    D.kv_gather(back, 256, 384, slots, kp, vp)
    assert torch.equal(back[:, 256:], qkv[:, 256:])


def test_sampling_distribution(dev):
    torch.manual_seed(2)
    V = 50
    logits = torch.randn(1, V, device=dev).repeat(4000, 1)
    temps = torch.full((4000,), 0.7, device=dev)
    seeds = torch.arange(4000, device=dev)
    tok, lp, ent = D.sample(logits, temps, seeds, 0)
    p = torch.softmax(logits[0].float() / 0.7, -1).cpu()
    freq = torch.bincount(tok.long().cpu(), minlength=V).float() / 4000
    assert (freq - p).abs().max() < 0.03
    torch.testing.assert_close(lp.cpu(), torch.log(p)[tok.long().cpu()], rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(ent.cpu()[0], -(p * p.log()).sum(), rtol=1e-3, atol=1e-3)
    g, _, _ = D.sample(logits[:3], torch.zeros(3, device=dev), seeds[:3], 0)
    assert (g.long() == logits[:3].argmax(-1)).all()


def test_engine_greedy_gpu(dev):
    from aiohttp.test_utils import TestClient, TestServer

    from agent_factory_3_b200.engine.scheduler import Engine
    from agent_factory_3_b200.engine.server import build_app
    from agent_factory_3_b200.models.gpt_oss import GptOssConfig, GptOssForCausalLM
    cfg = GptOssConfig(vocab_size=2048, hidden_size=256, intermediate_size=256, num_hidden_layers=2,
                       num_attention_heads=8, num_key_value_heads=2, head_dim=64,
                       num_local_experts=8, num_experts_per_tok=2, sliding_window=32,
                       rope_scaling=None, max_position_embeddings=4096, pad_token_id=0,
                       eos_token_id=1)
    model = GptOssForCausalLM(cfg, device=dev).init_random(0).eval()
    prompt = list(range(7, 207))
    eng = Engine(model, num_pages=128, page_size=64, max_prefill_tokens=96).start()

    async def run():
        c = TestClient(TestServer(build_app(eng)))
        await c.start_server()
        try:
            body = {"input_ids": prompt, "sampling_params": {"max_new_tokens": 8, "temperature": 0.0},
                    "return_routed_experts": True}
            a = await (await c.post("/generate", json=body)).json()
            b = await (await c.post("/generate", json=body)).json()
            return a, b
        finally:
            await c.close()

    try:
        a, b = asyncio.run(run())
    finally:
        eng.stop()
    # Teacher-forced check against a full recompute: a random-init model has near-tied logits
    # (top-2 gaps of a few 1e-3), so compare each greedy token with the recomputed logits at
    # its position instead of comparing token sequences.  Its router has near-ties too: the
    # recompute replays the experts the engine reported (R3), so a routing flip between the
    # decode path and the packed forward cannot move the logits.
    out = a["output_ids"]
    assert len(out) == 8, a
    ids = prompt + out[:-1]
    routed = np.frombuffer(base64.b64decode(a["meta_info"]["routed_experts"]), dtype=np.int32)
    routed = torch.from_numpy(routed.reshape(len(ids), cfg.num_hidden_layers,
                                             cfg.num_experts_per_tok).copy())
    with torch.no_grad():
        h = model.forward_hidden(torch.tensor(ids, device=dev), torch.arange(len(ids), device=dev),
                                 torch.tensor([0, len(ids)], dtype=torch.int32),
                                 routing_indices=routed.to(dev))
        lg = model.logits(h[len(prompt) - 1:]).float()
    chosen = lg[torch.arange(8, device=dev), torch.tensor(out, device=dev)]
    assert bool((chosen >= lg.max(-1).values - 0.05).all()), (out, lg.argmax(-1).tolist())
    assert b["output_ids"] == a["output_ids"]
    assert b["meta_info"]["cached_tokens"] >= 128


def test_mixed_adapter_step_gpu(dev):
    """Mixed-adapter step on the GPU kernels (masked dual GEMMs, MXFP4-direct experts with
    masked LoRA K blocks) against single-adapter steps."""
    from agent_factory_3_b200.engine.kv_cache import PagedKVCache
    from agent_factory_3_b200.engine.model_runner import ModelRunner, StepItem
    from agent_factory_3_b200.models.gpt_oss import GptOssConfig, GptOssForCausalLM, LoraConfig
    cfg = GptOssConfig(vocab_size=2048, hidden_size=256, intermediate_size=256, num_hidden_layers=2,
                       num_attention_heads=8, num_key_value_heads=2, head_dim=64,
                       num_local_experts=8, num_experts_per_tok=2, sliding_window=32,
                       rope_scaling=None, max_position_embeddings=4096, pad_token_id=0,
                       eos_token_id=1)
    lora = LoraConfig(r=16, lora_alpha=32, target_modules=["q_proj", "k_proj", "v_proj", "o_proj",
                                                           "gate_up_proj", "down_proj"])
    model = GptOssForCausalLM(cfg, lora=lora, device=dev).init_random(0).eval()
    params = model.lora_param_dict()
    bank = {}
    for name, seed in (("A", 1), ("B", 2)):
        g = torch.Generator(device=dev).manual_seed(seed)
        bank[name] = {k: (torch.randn(p.shape, generator=g, device=dev) * 0.05).to(torch.bfloat16)
                      for k, p in params.items()}
    prompts = {"A": list(range(3, 140)), "B": list(range(150, 171)), None: list(range(200, 213))}
    pages = {"A": [0, 1, 2], "B": [3], None: [4]}

    def kv():
        return PagedKVCache(2, 16, 64, 2, 64, 2, dev, torch.bfloat16)
    mixed = ModelRunner(model, kv()).forward_mixed(
        [StepItem(prompts[a], 0, pages[a], adapter=a) for a in ("A", "B", None)], bank).logits
    for j, a in enumerate(("A", "B", None)):
        if a is not None:
            with torch.no_grad():
                for k, p in params.items():
                    p.copy_(bank[a][k].float())
        ref = ModelRunner(model, kv(), lora_active=a is not None).forward(
            [StepItem(prompts[a], 0, pages[a])]).logits[0]
        err = (mixed[j] - ref).abs().max().item()
        assert err <= 0.02 * ref.abs().max().item() + 1e-3, (a, err)
