"""Rank-0-driven RPC over a Gloo group with 2 CPU ranks: broadcast calls, gathered reductions,
shutdown; and a rank that dies is reported as an error on the survivor (host-side fault
injection, no GPU involved)."""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from agent_factory_3_b200.parallel.rpc import RPCMixin, rpc_method


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class Worker(RPCMixin):
    def __init__(self):
        super().__init__()
        self.calls = []

    @rpc_method()
    def record(self, x):
        self.calls.append(x)
        return x

    @rpc_method(gather=True, reduce="mean_dict")
    def metric(self):
        return {"rank": float(dist.get_rank())}

    @rpc_method(gather=True, reduce="concat")
    def items(self):
        return [dist.get_rank()]


def _run(rank, port, q, die):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=20))
    w = Worker()
    try:
        if rank == 0:
            w.record(5)
            m = w.metric()
            it = w.items()
            if die:
                try:
                    w.record(6)   # rank 1 has exited: the broadcast must fail, not hang
                    w.record(7)
                    q.put(("no-error",))
                except Exception as e:  # noqa: BLE001
                    q.put(("error", type(e).__name__))
                return
            w.rpc_shutdown()
            q.put((w.calls, m, it))
        else:
            if die:
                # serve the first three calls, then leave without shutdown
                for _ in range(3):
                    name, args, kwargs, gather, reduce = w._rpc_broadcast(None)
                    w._rpc_run_local(name, args, kwargs, gather, reduce)
                os._exit(0)
            w.rpc_worker_loop()
            q.put(("r1", w.calls))
    finally:
        if not die:
            dist.destroy_process_group()


@pytest.mark.parametrize("die", [False, True])
def test_rpc_two_ranks(die):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_run, args=(r, port, q, die)) for r in range(2)]
    for p in ps:
        p.start()
    outs = [q.get(timeout=120) for _ in range(1 if die else 2)]
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    if die:
        assert outs[0][0] == "error"
    else:
        r0 = next(o for o in outs if o[0] != "r1")
        r1 = next(o for o in outs if o[0] == "r1")
        assert r0[0] == [5] and r1[1] == [5]
        assert r0[1] == {"rank": 0.5} and sorted(r0[2]) == [0, 1]


def test_payload_pack_roundtrip_keeps_arrays_as_views():
    import numpy as np

    from agent_factory_3_b200.parallel import payload
    from agent_factory_3_b200.trainer.types import TrainingSample
    rng = np.random.default_rng(1)
    s = TrainingSample(sample_id="a", input_ids=rng.integers(0, 1000, 37),
                       completion_mask=np.r_[np.zeros(5, np.int32), np.ones(32, np.int32)],
                       gen_logprobs=rng.normal(size=37).astype(np.float32),
                       advantages=np.ones(37, np.float32),
                       routing_indices=rng.integers(0, 128, (37, 3, 4)).astype(np.uint8),
                       seq_token_count=32, prompt_sequence_count=2, divisor=2.0)
    obj = ([s, s], [[0], [1]], {"k": None})
    buf = payload.pack(obj)
    back = payload.unpack(buf)
    assert back[1] == [[0], [1]] and back[2] == {"k": None}
    r = back[0][0]
    assert r.sample_id == "a" and r.divisor == 2.0
    for f in ("input_ids", "completion_mask", "gen_logprobs", "routing_indices"):
        a, b = getattr(s, f), getattr(r, f)
        assert a.dtype == b.dtype and np.array_equal(a, b)
        # a view of the buffer, at a 64-byte offset (so aligned for every dtype)
        assert np.shares_memory(b, buf) and (b.ctypes.data - buf.ctypes.data) % 64 == 0
        assert b.flags.aligned


def _scatter_rank(rank, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    import numpy as np

    from agent_factory_3_b200.parallel import payload
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=20))
    try:
        g = dist.new_group(backend="gloo")
        # payloads of different sizes; rank 0 keeps its own object as it is
        items = [("r0", np.arange(10, dtype=np.int64)), ("r1", np.arange(100000, dtype=np.float32))]
        got = payload.scatter(items if rank == 0 else None, group=g, src=0)
        q.put((rank, got[0], int(got[1].size), float(got[1].sum())))
    finally:
        dist.destroy_process_group()


def test_payload_scatter_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_scatter_rank, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(60)
    assert res[0] == (0, "r0", 10, 45.0)
    assert res[1][:3] == (1, "r1", 100000) and res[1][3] == float(np.arange(100000, dtype=np.float32).sum())
