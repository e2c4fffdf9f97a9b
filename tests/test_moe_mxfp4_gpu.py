"""MXFP4-direct (swap-AB) MoE expert GEMM on B200 against dequantise-then-GEMM in fp32:
every token tile size, both epilogues (clamped SwiGLU over interleaved gate/up rows, router-
gate row scale), expert LoRA as extra K blocks, experts with 0 and with more than 128 rows,
and rows outside the experts' valid ranges left untouched; then the whole inference MoE layer
against the training path."""
import pytest
import torch

from agent_factory_3_b200.ops import moe_layer, mxfp4
from agent_factory_3_b200.ops._ext import ext

pytestmark = pytest.mark.gpu


def _silu(g, u, alpha=1.702, limit=7.0):
    g = g.clamp(max=limit)
    u = u.clamp(-limit, limit)
    return g * torch.sigmoid(alpha * g) * (u + 1)


def _case(dev, E=6, N=256, K=192, r=0, seed=0):
    g = torch.Generator().manual_seed(seed)
    counts = torch.tensor([0, 3, 17, 40, 1, 130][:E], dtype=torch.int32)
    seg = (counts + 127) // 128 * 128
    offsets = torch.zeros(E + 1, dtype=torch.int32)
    offsets[1:] = torch.cumsum(seg, 0)
    R = int(offsets[-1])
    x = torch.randn(R, K, generator=g).bfloat16()
    blocks = torch.randint(0, 256, (E, N, K // 32, 16), generator=g, dtype=torch.uint8)
    scales = torch.randint(118, 126, (E, N, K // 32), generator=g, dtype=torch.uint8)
    bias = torch.randn(E, N, generator=g) * 0.1
    row_scale = torch.rand(R, generator=g)
    lb = (torch.randn(E, N, r, generator=g) * 0.05).bfloat16() if r else None
    xa = torch.randn(R, r, generator=g).bfloat16() if r else None
    W = mxfp4.dequantize_reference(blocks, scales).float()           # [E, N, K]
    pre = torch.zeros(R, N)
    valid = torch.zeros(R, dtype=torch.bool)
    for e in range(E):
        s0, n = int(offsets[e]), int(counts[e])
        if n == 0:
            continue
        y = x[s0:s0 + n].float() @ W[e].t() + bias[e]
        if r:
            y = y + xa[s0:s0 + n].float() @ lb[e].float().t()
        pre[s0:s0 + n] = y
        valid[s0:s0 + n] = True
    t = lambda v: None if v is None else v.to(dev)  # noqa: E731
    return dict(x=t(x), blocks=t(blocks), scales=t(scales), bias=t(bias), offsets=t(offsets),
                counts=t(counts), row_scale=t(row_scale), lb=t(lb), xa=t(xa)), pre, valid, row_scale


@pytest.mark.parametrize("bn", [16, 32, 64, 128])
@pytest.mark.parametrize("r", [0, 32])
@pytest.mark.parametrize("int_cvt", [0, 1])
def test_moe_mxfp4_gemm_matches_reference(dev, bn, r, int_cvt):
    d, pre, valid, row_scale = _case(dev, r=r, seed=bn + r)
    R, N = pre.shape
    out_sw = torch.full((R, N // 2), 7.0, device=dev, dtype=torch.bfloat16)
    ext().moe_mxfp4_gemm(d["x"], d["blocks"], d["scales"], d["bias"], d["offsets"], d["counts"], 0,
                         None, out_sw, 1.702, 7.0, bn, lora_b=d["lb"], xa=d["xa"], int_cvt=int_cvt)
    out_rs = torch.full((R, N), 7.0, device=dev, dtype=torch.bfloat16)
    ext().moe_mxfp4_gemm(d["x"], d["blocks"], d["scales"], d["bias"], d["offsets"], d["counts"], 1,
                         d["row_scale"], out_rs, 1.702, 7.0, bn, lora_b=d["lb"], xa=d["xa"],
                         int_cvt=int_cvt)
    torch.cuda.synchronize()
    assert ext().device_error() == 0
    q = pre.bfloat16().float()                      # the epilogue rounds gate/up to bf16 first
    ref_sw = _silu(q[:, 0::2], q[:, 1::2])
    ref_rs = row_scale[:, None] * pre
    got_sw, got_rs = out_sw.float().cpu(), out_rs.float().cpu()
    torch.testing.assert_close(got_sw[valid], ref_sw[valid], rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(got_rs[valid], ref_rs[valid], rtol=2e-2, atol=2e-2)
    assert bool((got_sw[~valid] == 7.0).all()) and bool((got_rs[~valid] == 7.0).all())


def test_inference_moe_layer_matches_training_path(dev, monkeypatch):
    from agent_factory_3_b200.models.gpt_oss import GptOssConfig, GptOssForCausalLM, LoraConfig
    cfg = GptOssConfig(vocab_size=512, hidden_size=256, intermediate_size=256, num_hidden_layers=1,
                       num_attention_heads=4, num_key_value_heads=2, head_dim=64,
                       num_local_experts=16, num_experts_per_tok=4, rope_scaling=None,
                       pad_token_id=0, eos_token_id=1)
    lora = LoraConfig(r=32, lora_alpha=64, target_modules=["gate_up_proj", "down_proj"])
    model = GptOssForCausalLM(cfg, lora=lora, device=dev).init_random(0)
    with torch.no_grad():
        for p in model.layers[0].mlp.lora.values():
            p.normal_(0, 0.02)
    mlp = model.layers[0].mlp
    xn = torch.randn(24, 256, device=dev).bfloat16()
    res = torch.randn(24, 256, device=dev).bfloat16()
    outs = {}
    for mode in ("0", "1"):
        monkeypatch.setenv("AF3_MOE_MXFP4", mode)
        with torch.no_grad():
            outs[mode] = mlp(xn, res).float()
    torch.testing.assert_close(outs["1"], outs["0"], rtol=3e-2, atol=3e-2)


def test_scale_range_guard(dev):
    """Scales outside [104, 140] are not exact in f16: the layer keeps the dequantise path."""
    from agent_factory_3_b200.ops.moe_layer import ExpertWeights, _mxfp4_direct
    E, N, K = 4, 64, 64
    b = torch.zeros(E, N, K // 32, 16, dtype=torch.uint8, device=dev)
    good = torch.full((E, N, K // 32), 120, dtype=torch.uint8, device=dev)
    ex = ExpertWeights(b, good, None, b[:, :, :], good, None)
    x = torch.zeros(8, K, device=dev).bfloat16()
    with torch.no_grad():
        assert _mxfp4_direct(x, ex, E, 2)
        bad = good.clone()
        bad[0, 0, 0] = 100
        assert not _mxfp4_direct(x, ExpertWeights(b, bad, None, b, good, None), E, 2)
        good[1, 1, 1] = 150          # in-place change: re-checked through the tensor version
        assert not _mxfp4_direct(x, ex, E, 2)


def test_integer_and_hardware_conversion_agree_bitwise(dev):
    """Both e2m1 -> f16 conversions are exact, so over every byte pattern and every scale the
    integer path allows (104..128) the two kernels must produce identical outputs."""
    g = torch.Generator().manual_seed(9)
    E, N, K, R = 2, 256, 512, 64
    blocks = torch.randint(0, 256, (E, N, K // 32, 16), generator=g, dtype=torch.uint8)
    scales = torch.randint(104, 129, (E, N, K // 32), generator=g, dtype=torch.uint8)
    x = (torch.randn(R, K, generator=g) * 0.5).bfloat16()
    offsets = torch.tensor([0, 32, 64], dtype=torch.int32)
    counts = torch.tensor([32, 32], dtype=torch.int32)
    row_scale = torch.rand(R, generator=g)
    outs = []
    for ic in (0, 1):
        o = torch.zeros(R, N, device=dev, dtype=torch.bfloat16)
        ext().moe_mxfp4_gemm(x.to(dev), blocks.to(dev), scales.to(dev), None, offsets.to(dev),
                             counts.to(dev), 1, row_scale.to(dev), o, 1.702, 7.0, 32, int_cvt=ic)
        outs.append(o)
    torch.cuda.synchronize()
    assert ext().device_error() == 0
    assert torch.equal(outs[0], outs[1])
