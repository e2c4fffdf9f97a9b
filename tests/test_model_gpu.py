"""The gpt-oss model on the GPU kernels against the same model on the CPU reference path,
plus the fused LoRA / log-prob operators."""
import pytest
import torch

from agent_factory_3_b200.models.gpt_oss import GptOssConfig, GptOssForCausalLM, LoraConfig
from agent_factory_3_b200.ops import gemm as G
from agent_factory_3_b200.ops.linear import lora_linear
from agent_factory_3_b200.ops.logprob import linear_logprob_entropy, logprob_entropy_reference

pytestmark = pytest.mark.gpu


def small_cfg():
    return GptOssConfig(vocab_size=4096, hidden_size=256, intermediate_size=256,
                        num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                        head_dim=64, num_local_experts=8, num_experts_per_tok=2,
                        sliding_window=32, rope_scaling=None, max_position_embeddings=4096,
                        pad_token_id=0, eos_token_id=1)


def test_dual_gemm(dev):
    torch.manual_seed(0)
    x = torch.randn(300, 256, device=dev).bfloat16()
    W = torch.randn(384, 256, device=dev).bfloat16()
    xa = torch.randn(300, 32, device=dev).bfloat16()
    B = torch.randn(384, 32, device=dev).bfloat16()
    y = G.matmul(x, W, a2=xa, b2=B)
    ref = G.matmul_reference(x.cpu(), W.cpu(), a2=xa.cpu(), b2=B.cpu())
    assert (y.cpu().float() - ref.float()).abs().max() < 2e-2 * ref.float().abs().max()


def test_lora_linear_grads(dev):
    torch.manual_seed(1)
    T, IN, OUT, r = 200, 256, 320, 16
    x = torch.randn(T, IN).bfloat16()
    W = (torch.randn(OUT, IN) * 0.05).bfloat16()
    b = torch.randn(OUT)
    A = torch.randn(r, IN) * 0.05
    B = torch.randn(OUT, r) * 0.05
    res = torch.randn(T, OUT).bfloat16()
    dy = torch.randn(T, OUT).bfloat16()
    outs = {}
    for d in ("cpu", dev):
        xx = x.to(d).float().requires_grad_(True) if d == "cpu" else x.to(d).requires_grad_(True)
        AA = A.detach().clone().to(d).requires_grad_(True)
        BB = B.detach().clone().to(d).requires_grad_(True)
        y = lora_linear(xx, W.to(d) if d != "cpu" else W.float(), b.to(d), AA, BB,
                        res.to(d) if d != "cpu" else res.float(), 2.0)
        y.backward(dy.to(d) if d != "cpu" else dy.float())
        outs[str(d)] = [t.detach().cpu().float() for t in (y, xx.grad, AA.grad, BB.grad)]
    for name, g, c in zip("y dx dA dB".split(), outs[str(dev)], outs["cpu"]):
        err = (g - c).abs().max().item()
        assert err <= 3e-2 * c.abs().max().item() + 1e-4, (name, err)


def test_linear_logprob(dev):
    torch.manual_seed(2)
    T, H, V = 300, 256, 1000
    h = torch.randn(T, H).bfloat16()
    W = (torch.randn(V, H) * 0.1).bfloat16()
    y = torch.randint(0, V, (T,))
    hg = h.to(dev).requires_grad_(True)
    lp, ent = linear_logprob_entropy(hg, W.to(dev), y.to(dev), temperature=0.7, chunk=384)
    g_lp, g_ent = torch.randn(T), torch.randn(T)
    (lp * g_lp.to(dev) + ent * g_ent.to(dev)).sum().backward()
    hr = h.float().requires_grad_(True)
    lp_r, ent_r = logprob_entropy_reference(hr, W.float(), y, 0.7)
    (lp_r * g_lp + ent_r * g_ent).sum().backward()
    torch.testing.assert_close(lp.cpu(), lp_r.detach(), rtol=1e-2, atol=2e-2)
    torch.testing.assert_close(ent.cpu(), ent_r.detach(), rtol=1e-2, atol=2e-2)
    err = (hg.grad.cpu().float() - hr.grad).abs().max().item()
    assert err <= 3e-2 * hr.grad.abs().max().item(), err


def test_model_gpu_matches_cpu(dev):
    cfg = small_cfg()
    lora = LoraConfig(r=16, lora_alpha=32, target_modules=["q_proj", "k_proj", "v_proj", "o_proj",
                                                            "gate_up_proj", "down_proj"])
    cpu = GptOssForCausalLM(cfg, lora, dtype=torch.float32).init_random(0)
    with torch.no_grad():
        for layer in cpu.layers:
            for name, p in list(layer.self_attn.lora.items()) + list(layer.mlp.lora.items()):
                if name.endswith("_B"):
                    p.normal_(0, 0.02)
    gpu = GptOssForCausalLM(cfg, lora, device=dev, dtype=torch.bfloat16)
    gpu.load_state_dict({k: v.to(dev) for k, v in cpu.state_dict().items()})
    with torch.no_grad():  # CPU oracle sees the bf16-rounded weights
        for (n, p) in cpu.named_parameters():
            if p.dtype == torch.float32 and "lora" not in n and p.dim() >= 2:
                p.copy_(p.bfloat16().float())
    seqlens = [300, 129, 75]
    g = torch.Generator().manual_seed(4)
    ids = torch.randint(0, cfg.vocab_size, (sum(seqlens),), generator=g)
    pos = torch.cat([torch.arange(n) for n in seqlens])
    cu = torch.tensor([0] + torch.tensor(seqlens).cumsum(0).tolist(), dtype=torch.int32)
    labels = torch.roll(ids, -1)
    with torch.no_grad():
        _, rec_cpu = cpu.forward_hidden(ids, pos, cu, record_routing=True)
    res = {}
    for name, m, d in (("cpu", cpu, "cpu"), ("gpu", gpu, dev)):
        m.gradient_checkpointing = True
        with torch.no_grad():
            _, rec = m.forward_hidden(ids.to(d), pos.to(d), cu, record_routing=True)
        # replay the same (CPU-recorded) routing on both sides
        h = m.forward_hidden(ids.to(d), pos.to(d), cu, routing_indices=rec_cpu.to(d))
        lp, ent = m.token_logprobs(h, labels.to(d))
        (-lp.sum()).backward()
        grads = {n: p.grad.detach().float().cpu() for n, p in m.named_parameters() if p.requires_grad}
        res[name] = (lp.detach().float().cpu(), rec.cpu(), grads)
    lp_c, rec_c, g_c = res["cpu"]
    lp_g, rec_g, g_g = res["gpu"]
    agree = (rec_c == rec_g).float().mean().item()
    assert agree > 0.97, agree
    err_lp = (lp_c - lp_g).abs().max().item()
    assert err_lp < 0.1, err_lp
    for n in g_c:
        err = (g_c[n] - g_g[n]).norm() / (g_c[n].norm() + 1e-8)
        assert err < 0.05, (n, err.item())


def test_attention_output_cache_gives_same_gradients(dev):
    """A checkpointed step that hands full-attention outputs to the recompute gives the same
    loss as one that recomputes every attention kernel, and LoRA gradients equal up to the
    run-to-run order of the backward's float atomics; the cache is used by the full layer."""
    from agent_factory_3_b200.ops.attention import AttentionOutputCache, AttentionPlan
    cfg = small_cfg()
    lora = LoraConfig(r=8, lora_alpha=16, target_modules=["q_proj", "o_proj", "gate_up_proj"])
    m = GptOssForCausalLM(cfg, lora=lora, device=dev).init_random(0).init_lora(1)
    with torch.no_grad():
        for p in m.lora_param_dict().values():
            p.normal_(0, 0.05)
    m.gradient_checkpointing = True
    T = 700
    g = torch.Generator().manual_seed(5)
    ids = torch.randint(0, cfg.vocab_size, (T,), generator=g).to(dev)
    pos = torch.cat([torch.arange(400), torch.arange(300)]).to(dev)
    cu = torch.tensor([0, 400, 700], dtype=torch.int32)
    labels = torch.roll(ids, -1)
    results = []
    for cache_bytes in (0, 1 << 30):
        plan = AttentionPlan(cu, dev)
        if cache_bytes:
            plan.cache = AttentionOutputCache(cache_bytes)
        for p in m.parameters():
            p.grad = None
        h = m.forward_hidden(ids, pos, cu, plan=plan)
        lp, _ = m.token_logprobs(h, labels)
        loss = -lp.sum()
        loss.backward()
        grads = [p.grad.detach().clone() for p in m.lora_param_dict().values()]
        results.append((loss.item(), grads, plan.cache))
    assert results[0][0] == results[1][0]
    cache = results[1][2]
    assert cache.hits == sum(1 for li in range(cfg.num_hidden_layers) if cfg.window(li) == 0)
    assert cache.used == 0 and not cache.entries
    for a, b in zip(results[0][1], results[1][1]):
        torch.testing.assert_close(a, b, rtol=1e-3, atol=1e-3 * float(a.abs().max()) + 1e-6)
