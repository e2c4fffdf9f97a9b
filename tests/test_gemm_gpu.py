"""tcgen05 GEMM numerics against the fp32 PyTorch reference of the same op."""
import pytest
import torch

from agent_factory_3_b200.ops import gemm as G

pytestmark = pytest.mark.gpu


def _close(x, ref, tol=2e-2):
    x = x.float().cpu()
    ref = ref.float().cpu()
    err = (x - ref).abs().max().item()
    scale = ref.abs().max().item() + 1e-6
    assert err <= tol * scale, f"max err {err} vs scale {scale}"


@pytest.mark.parametrize("M,N,K,bn", [(300, 384, 512, 256), (128, 256, 64, 128),
                                       (257, 96, 320, 32), (64, 200, 128, 64)])
def test_dense_nk(dev, M, N, K, bn):
    torch.manual_seed(0)
    a = torch.randn(M, K, device=dev).bfloat16()
    b = torch.randn(N, K, device=dev).bfloat16()
    bias = torch.randn(N, device=dev)
    y = G.matmul(a, b, bias=bias, bn=bn)
    _close(y, G.matmul_reference(a.cpu(), b.cpu(), bias=bias.cpu()))
    assert G.ext().device_error() == 0


def test_dense_fp32_accumulate_and_residual(dev):
    torch.manual_seed(1)
    a = torch.randn(200, 192, device=dev).bfloat16()
    b = torch.randn(128, 192, device=dev).bfloat16()
    out = torch.randn(200, 128, device=dev)
    ref = out.cpu() + a.cpu().float() @ b.cpu().float().t() * 0.5
    G.matmul(a, b, out=out, accumulate=True, alpha=0.5)
    _close(out, ref, 1e-3)
    res = torch.randn(200, 128, device=dev).bfloat16()
    y = G.matmul(a, b, residual=res)
    _close(y, G.matmul_reference(a.cpu(), b.cpu(), residual=res.cpu()))


@pytest.mark.parametrize("M,N,K", [(256, 320, 192), (130, 64, 128), (128, 32, 96)])
def test_dense_kn(dev, M, N, K):
    torch.manual_seed(2)
    a = torch.randn(M, K, device=dev).bfloat16()
    b = torch.randn(K, N, device=dev).bfloat16()
    y = G.matmul(a, b, b_layout="kn")
    _close(y, G.matmul_reference(a.cpu(), b.cpu(), b_layout="kn"))


@pytest.mark.parametrize("M,N,K", [(200, 256, 384), (32, 576, 256)])
def test_dense_km_kn(dev, M, N, K):
    torch.manual_seed(3)
    a = torch.randn(K, M, device=dev).bfloat16()
    b = torch.randn(K, N, device=dev).bfloat16()
    y = G.matmul(a, b, a_layout="km", b_layout="kn", out_dtype=torch.float32)
    _close(y, G.matmul_reference(a.cpu(), b.cpu(), "km", "kn", out_dtype=torch.float32), 1e-3)


def _segments(counts):
    offs = [0]
    for c in counts:
        offs.append(offs[-1] + (c + 127) // 128 * 128)
    return offs


@pytest.mark.parametrize("epi", ["bf16", "rowscale", "swiglu"])
def test_grouped_nk(dev, epi):
    torch.manual_seed(4)
    counts = [5, 0, 300, 128, 77]
    offs = _segments(counts)
    R, K, N, E = offs[-1], 192, 384, len(counts)
    a = torch.zeros(R, K, device=dev).bfloat16()
    for g, c in enumerate(counts):
        a[offs[g]:offs[g] + c] = torch.randn(c, K, device=dev).bfloat16()
    b = (torch.randn(E, N, K, device=dev) * 0.1).bfloat16()
    bias = torch.randn(E, N, device=dev)
    rs = torch.rand(R, device=dev)
    o = torch.tensor(offs, device=dev, dtype=torch.int32)
    out, out2 = G.grouped_matmul(a, b, o, epilogue=epi, bias=bias, row_scale=rs,
                                 save_preact=True)
    ref, ref2 = G.grouped_matmul_reference(a.cpu(), b.cpu(), o.cpu(), "nk", epi, bias.cpu(),
                                           rs.cpu())
    _close(out, ref)
    if epi == "swiglu":
        _close(out2, ref2)


def test_grouped_kn_swiglu_bwd(dev):
    torch.manual_seed(5)
    counts = [130, 3, 0, 256]
    offs = _segments(counts)
    R, K, N, E = offs[-1], 256, 192, len(counts)
    a = torch.randn(R, K, device=dev).bfloat16()
    b = (torch.randn(E, K, N, device=dev) * 0.1).bfloat16()
    aux = (torch.randn(R, 2 * N, device=dev) * 4).bfloat16()
    o = torch.tensor(offs, device=dev, dtype=torch.int32)
    out, _ = G.grouped_matmul(a, b, o, b_layout="kn", epilogue="swiglu_bwd", aux=aux)
    ref, _ = G.grouped_matmul_reference(a.cpu(), b.cpu(), o.cpu(), "kn", "swiglu_bwd",
                                        aux=aux.cpu())
    _close(out, ref, 3e-2)
    out_plain, _ = G.grouped_matmul(a, b, o, b_layout="kn", epilogue="bf16")
    ref_plain, _ = G.grouped_matmul_reference(a.cpu(), b.cpu(), o.cpu(), "kn", "bf16")
    _close(out_plain, ref_plain)


def test_grouped_k(dev):
    torch.manual_seed(6)
    counts = [128, 0, 384, 256]
    offs = _segments(counts)
    R = offs[-1]
    a = torch.randn(R, 32, device=dev).bfloat16()
    b = torch.randn(R, 320, device=dev).bfloat16()
    o = torch.tensor(offs, device=dev, dtype=torch.int32)
    out = G.grouped_k_matmul(a, b, o, alpha=0.25)
    _close(out, G.grouped_k_matmul_reference(a.cpu(), b.cpu(), o.cpu(), 0.25), 1e-3)
