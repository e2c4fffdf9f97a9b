"""Failure detection on the device without a GPU fault: kernels that wait for another rank give
up after a bounded time, record an error code in the device error word and return, the context
stays usable, and the host raises.  Here the "missing rank" is a flag that nothing writes, on
one GPU (no second process, no peer memory)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_fused_allreduce_times_out_on_a_missing_rank():
    from agent_factory_3_b200.ops._ext import check_device_error, ext
    dev = torch.device("cuda")
    assert ext().device_error() == 0
    T, H = 4, 256
    flags = torch.zeros(2, 64, dtype=torch.int32, device=dev)   # rank 0's and "rank 1's" flags
    parts = torch.randn(2, T, H, device=dev).to(torch.bfloat16)
    res = torch.randn(T, H, device=dev).to(torch.bfloat16)
    w = torch.ones(H, device=dev)
    x = torch.full((T, H), 7.0, device=dev).to(torch.bfloat16)
    xn = torch.empty_like(x)
    bufs = [parts[0].data_ptr(), parts[1].data_ptr()]
    fl = [flags[0].data_ptr(), flags[1].data_ptr()]
    ext().tp_allreduce_norm(bufs, fl, 0, 1, H, res, w, 1e-5, x, xn, T, H, 0.05)
    torch.cuda.synchronize()                     # returns: the wait was bounded
    with pytest.raises(RuntimeError, match="error code 2"):
        check_device_error()                      # kErrPeerTimeout, then cleared
    assert ext().device_error() == 0
    assert bool((x.float() == 7.0).all())         # nothing was written after the time-out
    # the context is still usable: the same kernel completes once "rank 1" has arrived
    flags[0, 1] = 1
    ext().tp_allreduce_norm(bufs, fl, 0, 1, H, res, w, 1e-5, x, xn, T, H, 0.05)
    torch.cuda.synchronize()
    assert ext().device_error() == 0
    want = (res.float() + parts.float().sum(0)).to(torch.bfloat16)
    torch.testing.assert_close(x.float(), want.float(), rtol=1e-2, atol=1e-2)


def test_gradient_reduction_times_out_on_a_missing_rank():
    from agent_factory_3_b200.ops._ext import ext
    dev = torch.device("cuda")
    S = 1024
    inbox = torch.randn(2 * S, device=dev)
    flags = torch.zeros(64, dtype=torch.int32, device=dev)
    flags[0] = 1                                  # rank 0 arrived, rank 1 never does
    out = torch.full((S,), 3.0, device=dev)
    sq = torch.zeros(1, device=dev)
    ext().grad_reduce(inbox.data_ptr(), flags.data_ptr(), 2, 1, out, sq, 0.05)
    torch.cuda.synchronize()
    assert ext().device_error() == 2
    assert bool((out == 3.0).all()) and float(sq) == 0.0
    flags[1] = 1
    ext().grad_reduce(inbox.data_ptr(), flags.data_ptr(), 2, 1, out, sq, 0.05)
    torch.cuda.synchronize()
    assert ext().device_error() == 0
    torch.testing.assert_close(out, inbox[:S] + inbox[S:])
    torch.testing.assert_close(sq, (out * out).sum().reshape(1), rtol=1e-5, atol=1e-3)


def test_tp_step_raises_on_device_error():
    """The tensor-parallel runner turns a recorded device error into a failed step."""
    from agent_factory_3_b200.engine.tp import TPContext
    ctx = TPContext.__new__(TPContext)
    ctx.rank, ctx.timeout_s = 0, 0.05
    from agent_factory_3_b200.ops._ext import ext
    dev = torch.device("cuda")
    flags = torch.zeros(2, 64, dtype=torch.int32, device=dev)
    parts = torch.zeros(2, 1, 256, device=dev).to(torch.bfloat16)
    x = torch.empty(1, 256, device=dev).to(torch.bfloat16)
    ext().tp_allreduce_norm([parts[0].data_ptr(), parts[1].data_ptr()],
                            [flags[0].data_ptr(), flags[1].data_ptr()], 0, 1, 256, None, None,
                            1e-5, x, None, 1, 256, 0.05)
    with pytest.raises(RuntimeError, match="did not arrive"):
        ctx.raise_on_device_error()
    assert ext().device_error() == 0
