"""FP8 (e4m3) expert mode on the CPU reference path: per-row quantisation error bound, exact
MXFP4 -> e4m3 conversion with an expert scale, and a model whose MoE layers run in fp8 staying
close to the bf16 model (loss, routing replayed, LoRA gradients)."""
import torch

from agent_factory_3_b200.models.gpt_oss import GptOssConfig, GptOssForCausalLM, LoraConfig
from agent_factory_3_b200.ops import fp8, mxfp4


def test_quant_rows_error_bound():
    torch.manual_seed(0)
    x = (torch.randn(7, 256) * torch.logspace(-3, 2, 7)[:, None]).bfloat16()
    x[3] = 0
    q, sc = fp8.quant_rows(x)
    back = fp8.e4m3_to_float(q) * sc[:, None]
    amax = x.float().abs().amax(1, keepdim=True)
    # 3 mantissa bits: half an ulp is 2^-4 relative; subnormals at 2^-9 of the row scale
    err = (back - x.float()).abs()
    assert bool((err <= x.float().abs() * 2 ** -4 + amax / 448 * 2 ** -9 + 1e-30).all())
    assert sc[3] == 1.0 and bool((q[3] == 0).all())


def test_mxfp4_to_e4m3_is_exact_with_expert_scale():
    torch.manual_seed(1)
    w = torch.randn(4, 16, 128) * torch.tensor([0.01, 0.1, 1.0, 10.0])[:, None, None]
    blocks, scales = mxfp4.quantize(w)
    w8, es = fp8.mxfp4_to_e4m3(blocks, scales)
    ref = mxfp4.dequantize(blocks, scales).float()
    assert torch.equal(fp8.e4m3_to_float(w8) * es[:, None, None], ref)
    wt = fp8.transpose_u8(w8)
    assert torch.equal(wt, w8.transpose(1, 2))


def _cfg():
    return GptOssConfig(vocab_size=1024, hidden_size=256, intermediate_size=256,
                        num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                        head_dim=64, num_local_experts=8, num_experts_per_tok=2,
                        sliding_window=32, rope_scaling=None, max_position_embeddings=2048,
                        pad_token_id=0, eos_token_id=1)


def test_fp8_moe_model_close_to_bf16():
    cfg = _cfg()
    lora = LoraConfig(r=8, lora_alpha=16, target_modules=["q_proj", "o_proj", "gate_up_proj",
                                                          "down_proj"])
    model = GptOssForCausalLM(cfg, lora, dtype=torch.float32).init_random(0)
    with torch.no_grad():
        for layer in model.layers:
            for name, p in layer.mlp.lora.items():
                if name.endswith("_B"):
                    p.normal_(0, 0.02)
    g = torch.Generator().manual_seed(2)
    ids = torch.randint(2, cfg.vocab_size, (160,), generator=g)
    pos = torch.arange(160)
    cu = torch.tensor([0, 160], dtype=torch.int32)
    labels = torch.roll(ids, -1)
    with torch.no_grad():
        _, rec = model.forward_hidden(ids, pos, cu, record_routing=True)
    res = {}
    for mode in ("bf16", "fp8"):
        for layer in model.layers:
            layer.mlp.dequant_dtype = mode
        model.zero_grad(set_to_none=True)
        h = model.forward_hidden(ids, pos, cu, routing_indices=rec)
        lp, _ = model.token_logprobs(h, labels)
        (-lp.sum()).backward()
        res[mode] = (lp.detach().clone(), {n: p.grad.detach().clone()
                                           for n, p in model.named_parameters()
                                           if p.requires_grad and p.grad is not None})
    lp_b, g_b = res["bf16"]
    lp_f, g_f = res["fp8"]
    assert (lp_b - lp_f).abs().mean() < 0.05 * lp_b.abs().mean()
    checked = 0
    for n in g_b:
        if g_b[n].norm() == 0:          # A factors under zero-initialised B factors
            assert g_f[n].norm() == 0, n
            continue
        cos = torch.nn.functional.cosine_similarity(g_b[n].flatten(), g_f[n].flatten(), dim=0)
        assert cos > 0.98, (n, cos.item())
        checked += 1
    assert checked >= 4
