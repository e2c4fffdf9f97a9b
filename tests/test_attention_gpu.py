"""sm_100a flash attention (sinks, sliding window, packed varlen, GQA) against the dense fp32
reference of the same op."""
import math

import pytest
import torch

from agent_factory_3_b200.ops import attention as A

pytestmark = pytest.mark.gpu

CASES = [
    ([300], 0), ([300, 129, 75, 1], 0), ([300, 129, 75, 1], 32), ([517], 128), ([64, 700], 128),
    ([2048, 300], 0),   # many unmasked blocks: the FMA-pipe exponentials and lazy rescaling
]


def _inputs(seqlens, hq=8, hkv=2, d=64, seed=0):
    g = torch.Generator().manual_seed(seed)
    T = sum(seqlens)
    qkv = (torch.randn(T, (hq + 2 * hkv) * d, generator=g)).bfloat16()
    sinks = torch.randn(hq, generator=g)
    cu = torch.tensor([0] + torch.tensor(seqlens).cumsum(0).tolist(), dtype=torch.int32)
    return qkv, sinks, cu


@pytest.mark.parametrize("seqlens,window", CASES)
def test_attn_fwd(dev, seqlens, window):
    hq, hkv, d = 8, 2, 64
    qkv, sinks, cu = _inputs(seqlens, hq, hkv, d)
    ref, lse_ref = A.attention_reference(qkv.float(), cu, sinks, hq, hkv, d, window,
                                         return_lse=True)
    plan = A.AttentionPlan(cu, dev)
    out = torch.empty(qkv.shape[0], hq * d, device=dev, dtype=torch.bfloat16)
    lse = torch.empty(hq, qkv.shape[0], device=dev, dtype=torch.float32)
    A.ext().attn_fwd(qkv.to(dev), sinks.to(dev), plan.tiles, plan.cu, out, lse, hq, hkv, d,
                     window, 1.0 / math.sqrt(d))
    torch.cuda.synchronize()
    assert A.ext().device_error() == 0
    err = (out.cpu().float() - ref).abs().max().item()
    assert err < 2e-2, err
    torch.testing.assert_close(lse.cpu(), lse_ref, rtol=1e-3, atol=2e-3)


@pytest.mark.parametrize("window", [0, 32])
def test_attn_fwd_large_scores(dev, window):
    """Scores far above and below the sinks: early rows whose visible scores all lie far below
    the sink must stay finite (the sink joins the row max)."""
    hq, hkv, d, L = 8, 2, 64, 300
    qkv, sinks, cu = _inputs([L], hq, hkv, d, seed=3)
    qkv = (qkv.float() * 8).bfloat16()
    ref, lse_ref = A.attention_reference(qkv.float(), cu, sinks, hq, hkv, d, window, return_lse=True)
    plan = A.AttentionPlan(cu, dev)
    out = torch.empty(L, hq * d, device=dev, dtype=torch.bfloat16)
    lse = torch.empty(hq, L, device=dev, dtype=torch.float32)
    A.ext().attn_fwd(qkv.to(dev), sinks.to(dev), plan.tiles, plan.cu, out, lse, hq, hkv, d,
                     window, 1.0 / math.sqrt(d))
    torch.cuda.synchronize()
    assert bool(torch.isfinite(lse).all()) and bool(torch.isfinite(out.float()).all())
    torch.testing.assert_close(lse.cpu(), lse_ref, rtol=1e-3, atol=5e-3)
    err = (out.cpu().float() - ref).abs().max().item()
    assert err < 0.15, err   # |v| ~ 8: a few bf16 ulps


@pytest.mark.parametrize("seqlens,window", CASES)
def test_attn_fwd_bwd(dev, seqlens, window):
    hq, hkv, d = 8, 2, 64
    qkv, sinks, cu = _inputs(seqlens, hq, hkv, d, seed=1)
    dout = torch.randn(qkv.shape[0], hq * d).bfloat16()
    x = qkv.float().requires_grad_(True)
    sk = sinks.clone().requires_grad_(True)
    ref = A.attention_reference(x, cu, sk, hq, hkv, d, window)
    ref.backward(dout.float())
    xg = qkv.to(dev).requires_grad_(True)
    sg = sinks.to(dev).requires_grad_(True)
    out = A.attention(xg, sg, cu, hq, hkv, d, window)
    out.backward(dout.to(dev))
    torch.cuda.synchronize()
    assert A.ext().device_error() == 0
    assert (out.detach().cpu().float() - ref.detach()).abs().max().item() < 2e-2
    gq = xg.grad.cpu().float()
    for name, sl in (("dq", slice(0, hq * d)), ("dk", slice(hq * d, (hq + hkv) * d)),
                     ("dv", slice((hq + hkv) * d, None))):
        err = (gq[:, sl] - x.grad[:, sl]).abs().max().item()
        scale = x.grad[:, sl].abs().max().item()
        assert err <= 2e-2 * scale + 1e-3, (name, err, scale)
    torch.testing.assert_close(sg.grad.cpu(), sk.grad, rtol=2e-2, atol=2e-2)
