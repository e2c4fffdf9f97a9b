"""Rank-0-driven RPC over a Gloo group with 2 CPU ranks: broadcast calls, gathered reductions,
shutdown; and a rank that dies is reported as an error on the survivor (host-side fault
injection, no GPU involved)."""
import os
import socket

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
