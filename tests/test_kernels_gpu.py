"""MoE plumbing, MXFP4 codec and memory-bound kernels against PyTorch fp32 references."""
import pytest
import torch

from agent_factory_3_b200.ops import activation, moe, mxfp4, norm, rope

pytestmark = pytest.mark.gpu


def test_mxfp4_dequant_bit_exact(dev):
    torch.manual_seed(0)
    blocks = torch.randint(0, 256, (4, 96, 5, 16), dtype=torch.uint8)
    scales = torch.randint(100, 150, (4, 96, 5), dtype=torch.uint8)
    ref = mxfp4.dequantize_reference(blocks, scales)
    out = mxfp4.dequantize(blocks.to(dev), scales.to(dev))
    assert torch.equal(out.cpu().view(torch.int16), ref.view(torch.int16))


def test_mxfp4_dequant_exhaustive(dev):
    """Every packed byte under every finite e8m0 scale (0 = 2^-127 .. 254), bit for bit."""
    s = torch.arange(255, dtype=torch.uint8)
    blocks = torch.arange(256, dtype=torch.int64).to(torch.uint8).view(1, 16, 16).repeat(255, 1, 1)
    scales = s.view(255, 1).repeat(1, 16)
    ref = mxfp4.dequantize_reference(blocks, scales)
    out = mxfp4.dequantize(blocks.to(dev), scales.to(dev))
    assert torch.equal(out.cpu().view(torch.int16), ref.view(torch.int16))


@pytest.mark.parametrize("replay", [False, True])
def test_route_and_group(dev, replay):
    torch.manual_seed(1)
    T, E, K = 3000, 32, 4
    logits = torch.randn(T, E)
    ids = None
    if replay:
        ids = torch.stack([torch.randperm(E)[:K] for _ in range(T)]).to(torch.int32)
    ref_ids, ref_g = moe.route_reference(logits, K, ids)
    ref = moe.group_reference(ref_ids, ref_g, E)
    r = moe.route(logits.to(dev), K, E, replay_ids=None if ids is None else ids.to(dev))
    assert torch.equal(r.ids.cpu(), ref.ids)
    torch.testing.assert_close(r.gates.cpu(), ref.gates, rtol=1e-5, atol=1e-6)
    assert torch.equal(r.offsets.cpu(), ref.offsets)
    assert torch.equal(r.dest.cpu(), ref.dest)
    assert torch.equal(r.row_src.cpu(), ref.row_src)


def test_gather_combine(dev):
    torch.manual_seed(2)
    T, E, K, H = 500, 8, 2, 256
    x = torch.randn(T, H).bfloat16()
    ids, gates = moe.route_reference(torch.randn(T, E), K)
    rt = moe.group_reference(ids, gates, E)
    xs = moe.gather_rows(x.to(dev), rt.row_src.to(dev), rt.row_gate.to(dev))
    xs_ref = moe.gather_rows(x, rt.row_src, rt.row_gate)
    torch.testing.assert_close(xs.cpu().float(), xs_ref.float(), rtol=1e-2, atol=1e-2)
    res = torch.randn(T, H).bfloat16()
    y = moe.combine_rows(xs, rt.dest.to(dev), K, residual=res.to(dev))
    y_ref = moe.combine_rows(xs_ref, rt.dest, K, residual=res)
    torch.testing.assert_close(y.cpu().float(), y_ref.float(), rtol=2e-2, atol=2e-2)


def test_rmsnorm(dev):
    torch.manual_seed(3)
    x = torch.randn(333, 2880).bfloat16()
    w = torch.rand(2880) + 0.5
    y, rstd = norm.rmsnorm_fwd(x.to(dev), w.to(dev), 1e-5)
    torch.testing.assert_close(y.cpu().float(), norm.rmsnorm_reference(x, w, 1e-5).float(),
                               rtol=1e-2, atol=1e-2)
    dy = torch.randn(333, 2880).bfloat16()
    dx, dw = norm.rmsnorm_bwd(x.to(dev), w.to(dev), dy.to(dev), rstd, need_dw=True)
    xf = x.float().requires_grad_(True)
    wf = w.clone().requires_grad_(True)
    yr = wf * (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-5))
    gx, gw = torch.autograd.grad(yr, [xf, wf], dy.float())
    torch.testing.assert_close(dx.cpu().float(), gx, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(dw.cpu(), gw, rtol=1e-3, atol=1e-2)


def test_rope(dev):
    torch.manual_seed(4)
    cos, sin = rope.rope_tables(64, 4096, 150000.0, {"rope_type": "yarn", "factor": 32.0,
                                                       "original_max_position_embeddings": 4096,
                                                       "beta_fast": 32.0, "beta_slow": 1.0,
                                                       "truncate": False})
    T, nh = 100, 6
    qkv = torch.randn(T, (nh + 2) * 64).bfloat16()
    pos = torch.randint(0, 4096, (T,))
    ref = qkv.clone()
    rope.apply_rope_(ref, nh, 64, pos, cos, sin)
    out = qkv.to(dev)
    rope.apply_rope_(out, nh, 64, pos.to(dev), cos.to(dev), sin.to(dev))
    torch.testing.assert_close(out.cpu().float(), ref.float(), rtol=1e-2, atol=1e-2)
    # inverse rotation (backward): compare with the reference of the same op
    rope.apply_rope_(out, nh, 64, pos.to(dev), cos.to(dev), sin.to(dev), inverse=True)
    rope.apply_rope_(ref, nh, 64, pos, cos, sin, inverse=True)
    torch.testing.assert_close(out.cpu().float(), ref.float(), rtol=2e-2, atol=2e-2)


def test_swiglu(dev):
    torch.manual_seed(5)
    gu = (torch.randn(64, 512) * 5).bfloat16()
    h = activation.swiglu_fwd(gu.to(dev))
    torch.testing.assert_close(h.cpu().float(), activation.swiglu_fwd(gu).float(), rtol=1e-2,
                               atol=1e-2)
    d = torch.randn(64, 256).bfloat16()
    dg = activation.swiglu_bwd(gu.to(dev), d.to(dev))
    torch.testing.assert_close(dg.cpu().float(), activation.swiglu_bwd(gu, d).float(), rtol=2e-2,
                               atol=2e-2)
