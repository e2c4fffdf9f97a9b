"""GPU test of the allocation-free C entry point ``af3_decode_attention_noalloc``.

The entry point is called through its exported C symbol (ctypes on the in-tree extension
library) and must match the torch entry point ``decode_attention`` on two calls in a row, the
second reusing the device scratch the first one set up.  Oversize inputs must be rejected with
a message and without touching the output.  The file name sorts last so the test also runs
after every other test in a full session; it passes alone in a fresh process as well.
The C prototypes these ctypes signatures mirror are declared in
``csrc/decode_attention_noalloc.h``; a CPU test checks that the two agree."""
import ctypes
import math
import os
import re

import pytest
import torch

_P = ctypes.c_void_p
_I = ctypes.c_int
_LL = ctypes.c_longlong
_ARGTYPES = [_P, _LL, _P, _P, _P, _I, _P, _P, _P, _LL, _P, _I, _I, _I, _I, _I,
             ctypes.c_float, _I, _P]
_HEADER = os.path.join(os.path.dirname(__file__), "..", "agent_factory_3_b200", "csrc",
                       "decode_attention_noalloc.h")


def _ctype_of(decl: str):
    """ctypes type of one C parameter declaration of the header."""
    decl = decl.strip()
    if "*" in decl or decl.startswith("cudaStream_t"):
        return _P
    base = re.sub(r"\s+\w+$", "", decl)   # drop the parameter name
    return {"int": _I, "long long": _LL, "float": ctypes.c_float}[base]


def test_header_prototype_matches_ctypes_signature():
    text = open(_HEADER).read()
    m = re.search(r"int af3_decode_attention_noalloc\(([^)]*)\);", text)
    assert m, "prototype missing from the header"
    params = [p for p in m.group(1).replace("\n", " ").split(",")]
    assert [_ctype_of(p) for p in params] == _ARGTYPES
    for name, ret in (("af3_decode_attention_noalloc_scratch_bytes", "size_t"),
                      ("af3_decode_attention_noalloc_last_error", "const char*"),
                      ("af3_decode_attention_noalloc_init", "int")):
        assert re.search(rf"{re.escape(ret)} {name}\(void\);", text), name
    for code, val in (("OK", 0), ("INVALID_ARGUMENT", 1), ("TOO_LARGE", 2), ("CUDA_ERROR", 3)):
        assert re.search(rf"#define AF3_NOALLOC_{code} {val}\b", text), code


def _lib():
    import agent_factory_3_b200._C as C
    lib = ctypes.CDLL(C.__file__)
    f = lib.af3_decode_attention_noalloc
    f.restype = _I
    f.argtypes = _ARGTYPES
    lib.af3_decode_attention_noalloc_last_error.restype = ctypes.c_char_p
    lib.af3_decode_attention_noalloc_scratch_bytes.restype = ctypes.c_size_t
    lib.af3_decode_attention_noalloc_init.restype = _I
    return lib


def _inputs(dev, B=6, hq=64, hkv=8, P=64, max_pages=40):
    g = torch.Generator().manual_seed(7)
    pages = B * max_pages
    kp = torch.randn(pages, P, hkv, 64, generator=g).bfloat16().to(dev)
    vp = torch.randn(pages, P, hkv, 64, generator=g).bfloat16().to(dev)
    lens = torch.tensor([1, 63, 64, 700, 1500, 2500][:B], dtype=torch.int32)
    perm = torch.randperm(pages, generator=g)
    pt = torch.zeros(B, max_pages, dtype=torch.int32)
    for b in range(B):
        pt[b] = perm[b * max_pages:(b + 1) * max_pages]
    # q as a strided view of a wider row (like the q part of a packed qkv buffer)
    qkv = torch.randn(B, (hq + 2 * hkv) * 64, generator=g).bfloat16().to(dev)
    q = qkv[:, :hq * 64]
    sinks = torch.randn(hq, generator=g).to(dev)
    return q, kp, vp, pt.to(dev), lens.to(dev), sinks, int(lens.max())


def _call(lib, q, kp, vp, pt, lens, sinks, out, lse, hq, hkv, window, scale, msl):
    B = q.shape[0]
    return lib.af3_decode_attention_noalloc(
        q.data_ptr(), q.stride(0), kp.data_ptr(), vp.data_ptr(), pt.data_ptr(), pt.shape[1],
        lens.data_ptr(), sinks.data_ptr(), out.data_ptr(), out.stride(0),
        lse.data_ptr() if lse is not None else None, B, hq, hkv, kp.shape[1], window, scale, msl,
        torch.cuda.current_stream().cuda_stream)


@pytest.mark.gpu
@pytest.mark.parametrize("window", [0, 128])
def test_noalloc_matches_torch_entry_point(window):
    from agent_factory_3_b200.ops._ext import ext
    dev = torch.device("cuda")
    lib = _lib()
    hq, hkv = 64, 8
    q, kp, vp, pt, lens, sinks, msl = _inputs(dev, hq=hq, hkv=hkv)
    B = q.shape[0]
    scale = 1.0 / math.sqrt(64)
    ref = torch.empty(B, hq * 64, device=dev, dtype=torch.bfloat16)
    ref_lse = torch.empty(B, hq, device=dev, dtype=torch.float32)
    ext().decode_attention(q, kp, vp, pt, lens, sinks, ref, ref_lse, hq, hkv, window, scale, msl)
    assert lib.af3_decode_attention_noalloc_init() == 0
    for _ in range(2):   # second call reuses the scratch set up by the first
        out = torch.full((B, hq * 64), float("nan"), device=dev, dtype=torch.bfloat16)
        lse = torch.full((B, hq), float("nan"), device=dev, dtype=torch.float32)
        allocated = torch.cuda.memory_allocated(dev)
        rc = _call(lib, q, kp, vp, pt, lens, sinks, out, lse, hq, hkv, window, scale, msl)
        assert rc == 0, lib.af3_decode_attention_noalloc_last_error()
        torch.cuda.synchronize()
        assert torch.cuda.memory_allocated(dev) == allocated
        torch.testing.assert_close(out.float(), ref.float(), rtol=1e-2, atol=1e-2)
        torch.testing.assert_close(lse, ref_lse, rtol=1e-4, atol=1e-4)
    assert lib.af3_decode_attention_noalloc_last_error() == b""


@pytest.mark.gpu
def test_noalloc_rejects_oversize():
    dev = torch.device("cuda")
    lib = _lib()
    cap = lib.af3_decode_attention_noalloc_scratch_bytes()
    assert cap == 16 << 20
    hq, hkv = 64, 8
    q, kp, vp, pt, lens, sinks, _ = _inputs(dev, hq=hq, hkv=hkv)
    B = q.shape[0]
    # chunks needed so that B * hq * chunks * 66 floats exceed the scratch
    chunk_tokens = 16 * kp.shape[1]
    chunks = cap // (B * hq * 66 * 4) + 1
    msl = chunks * chunk_tokens
    big_pt = torch.zeros(B, chunks * 16, dtype=torch.int32, device=dev)
    out = torch.zeros(B, hq * 64, device=dev, dtype=torch.bfloat16)
    rc = _call(lib, q, kp, vp, big_pt, lens, sinks, out, None, hq, hkv, 0, 0.125, msl)
    torch.cuda.synchronize()
    assert rc == 2
    msg = lib.af3_decode_attention_noalloc_last_error().decode()
    assert "scratch" in msg and "split the batch" in msg
    assert bool((out == 0).all())
    # an unsupported head grouping is an argument error, also before any launch
    rc = _call(lib, q, kp, vp, pt, lens, sinks, out, None, 48, 8, 0, 0.125, 64)
    assert rc == 1 and b"GQA group" in lib.af3_decode_attention_noalloc_last_error()


@pytest.mark.gpu
def test_noalloc_rejects_misaligned_operands():
    """Operands the kernels would read with 16-byte loads are checked on the host: a bad
    stride or pointer returns AF3_NOALLOC_INVALID_ARGUMENT and launches nothing."""
    dev = torch.device("cuda")
    lib = _lib()
    hq, hkv = 64, 8
    q, kp, vp, pt, lens, sinks, msl = _inputs(dev, hq=hq, hkv=hkv)
    B = q.shape[0]
    out = torch.zeros(B, hq * 64, device=dev, dtype=torch.bfloat16)
    stream = torch.cuda.current_stream().cuda_stream

    def call(q_ptr, ld_q, k_ptr, ld_out):
        return lib.af3_decode_attention_noalloc(
            q_ptr, ld_q, k_ptr, vp.data_ptr(), pt.data_ptr(), pt.shape[1], lens.data_ptr(),
            sinks.data_ptr(), out.data_ptr(), ld_out, None, B, hq, hkv, kp.shape[1], 0, 0.125,
            msl, stream)

    ld = q.stride(0)
    assert call(q.data_ptr(), ld + 1, kp.data_ptr(), out.stride(0)) == 1          # odd ld_q
    assert b"ld_q" in lib.af3_decode_attention_noalloc_last_error()
    assert call(q.data_ptr() + 2, ld, kp.data_ptr(), out.stride(0)) == 1          # q off by 2 B
    assert call(q.data_ptr(), ld, kp.data_ptr() + 8, out.stride(0)) == 1          # k off by 8 B
    assert b"16-byte" in lib.af3_decode_attention_noalloc_last_error()
    assert call(q.data_ptr(), hq * 64 - 8, kp.data_ptr(), out.stride(0)) == 1     # rows overlap
    assert call(q.data_ptr(), ld, kp.data_ptr(), hq * 64 - 1) == 1                # short out rows
    torch.cuda.synchronize()
    assert bool((out == 0).all())
