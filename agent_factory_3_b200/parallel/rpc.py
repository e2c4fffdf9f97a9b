"""Single-controller RPC over a CPU (Gloo) process group.

Rank 0 calls methods decorated with ``@rpc_method``; the call (method name, args, kwargs) is
pickled and broadcast to every other rank, which sits in ``rpc_worker_loop`` executing the
same method so collectives inside it line up.  Results can be gathered and reduced
("rank0", "mean_dict", "concat", "merge_dict", "mean_list_dict").  With one process, or when
torch.distributed is not initialised, calls run locally.  (Reference:
trainer/accelerate_rpc_mixin.py:38-428.)

The control group has a finite timeout (default 30 min, ``AF3_RPC_TIMEOUT_S``) so a dead rank
ends the job with an error instead of a silent hang; the reference uses 6 h.
"""
from __future__ import annotations

import datetime
import functools
import logging
import os
from typing import Any, Callable

import torch
import torch.distributed as dist

logger = logging.getLogger(__name__)

_SHUTDOWN = "__rpc_shutdown__"


def _reduce(results: list, mode: str):
    if mode == "rank0":
        return results[0]
    if mode == "concat":
        out = []
        for r in results:
            out.extend(r or [])
        return out
    if mode == "merge_dict":
        out = {}
        for r in results:
            out.update(r or {})
        return out
    if mode == "mean_dict":
        keys = set().union(*[r.keys() for r in results if r])
        return {k: sum(r[k] for r in results if r and k in r) /
                max(1, sum(1 for r in results if r and k in r)) for k in keys}
    if mode == "mean_list_dict":
        n = max(len(r or []) for r in results)
        return [_reduce([r[i] for r in results if r and i < len(r)], "mean_dict") for i in range(n)]
    raise ValueError(f"unknown reduce mode {mode!r}")


def rpc_method(gather: bool = False, reduce: str = "rank0"):
    """Decorator: when called on rank 0 of a distributed job, broadcast the call to the other
    ranks first; with ``gather`` the per-rank results are all-gathered and reduced."""

    def deco(fn: Callable):
        @functools.wraps(fn)
        def wrapper(self, *args, **kwargs):
            if getattr(self, "_rpc_executing", False) or not self._rpc_active():
                return fn(self, *args, **kwargs)
            return self._rpc_invoke(fn.__name__, args, kwargs, gather, reduce)

        wrapper._rpc_fn = fn
        wrapper._rpc_gather = gather
        wrapper._rpc_reduce = reduce
        return wrapper

    return deco


class RPCMixin:
    def __init__(self, group=None):
        self._rpc_group = group
        self._rpc_executing = False
        if group is None and dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
            backend = dist.get_backend()
            if backend == "gloo":
                self._rpc_group = dist.group.WORLD
            else:
                timeout = datetime.timedelta(seconds=float(os.environ.get("AF3_RPC_TIMEOUT_S", 1800)))
                self._rpc_group = dist.new_group(backend="gloo", timeout=timeout)

    def _rpc_active(self) -> bool:
        return (self._rpc_group is not None and dist.is_available() and dist.is_initialized()
                and dist.get_world_size() > 1)

    def _rpc_broadcast(self, obj):
        box = [obj]
        dist.broadcast_object_list(box, src=0, group=self._rpc_group)
        return box[0]

    def _rpc_run_local(self, name, args, kwargs, gather, reduce):
        method = getattr(type(self), name)
        fn = getattr(method, "_rpc_fn", method)
        self._rpc_executing = True
        try:
            result = fn(self, *args, **kwargs)
        finally:
            self._rpc_executing = False
        if not gather:
            return result
        out = [None] * dist.get_world_size()
        dist.all_gather_object(out, result, group=self._rpc_group)
        return _reduce(out, reduce)

    def _rpc_invoke(self, name, args, kwargs, gather, reduce):
        if dist.get_rank() != 0:
            raise RuntimeError(f"rpc method {name} must be called on rank 0 (others run rpc_worker_loop)")
        self._rpc_broadcast((name, args, kwargs, gather, reduce))
        return self._rpc_run_local(name, args, kwargs, gather, reduce)

    def rpc_worker_loop(self) -> None:
        """Ranks != 0: execute broadcast calls until ``rpc_shutdown``."""
        if not self._rpc_active():
            return
        while True:
            name, args, kwargs, gather, reduce = self._rpc_broadcast(None)
            if name == _SHUTDOWN:
                return
            self._rpc_run_local(name, args, kwargs, gather, reduce)

    def rpc_shutdown(self) -> None:
        if self._rpc_active() and dist.get_rank() == 0:
            self._rpc_broadcast((_SHUTDOWN, (), {}, False, "rank0"))
