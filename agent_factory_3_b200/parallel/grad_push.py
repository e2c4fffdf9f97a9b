"""Data-parallel reduce-scatter of the flat LoRA gradient, overlapped with the backward pass
(the reference reduces with FSDP2's NCCL reduce-scatter after the last microbatch's backward,
``trainer/model_trainer.py:505-510``).

Layout: the trainer keeps every trainable tensor's gradient in one flat fp32 buffer; with the
sharded optimizer, rank r owns the slice [r*S, (r+1)*S).  Each rank allocates an inbox that all
ranks map (``PeerMappedBuffer``): a 256-byte flag area and W slots of S floats, slot j receiving
rank j's contribution to this rank's slice.

Per step (``arm`` before the last microbatch's backward, ``finish`` after it):
  * a post-accumulate-grad hook fires when a parameter's gradient is final; its flat range is
    split by owner and each piece is copied into the owner's inbox slot with one async copy on
    a side stream (copy engines over NVLink, no SM time), after the side stream waited for the
    compute stream -- the transfer of early layers overlaps the backward of later ones;
  * ``finish`` copies the ranges no hook covered (tensors that got no gradient this step), then
    signals the owners (``grad_signal``), and the compute stream runs ``grad_reduce``, which
    waits (bounded) for every rank's signal and sums the W slots in rank order into the local
    shard gradient, returning its sum of squares for the global gradient norm.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops._ext import check_device_error, ext
from .symm import PeerMappedBuffer

FLAG_BYTES = 256


class GradientPusher:
    def __init__(self, params: list[torch.Tensor], offsets: list[int], flat_grad: torch.Tensor,
                 shard_grad: torch.Tensor, group=None, timeout_s: float = 600.0):
        self.group = group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        self.flat_grad, self.shard_grad = flat_grad, shard_grad
        self.S = shard_grad.numel()
        if flat_grad.numel() != self.S * self.world:
            raise ValueError("flat gradient must be world x shard size")
        self.timeout_s = timeout_s
        dev = flat_grad.device
        self.buf = PeerMappedBuffer(FLAG_BYTES + self.world * self.S * 4, group, dev)
        self.side = torch.cuda.Stream(device=dev)
        self.epoch = 0
        self.armed = False
        self.sumsq = torch.zeros(1, device=dev, dtype=torch.float32)
        # flat ranges [a, b) of every trainable tensor
        self.ranges = [(off, off + p.numel()) for p, off in zip(params, offsets)]
        self.pushed: list[bool] = [False] * len(params)
        self.hooks = [p.register_post_accumulate_grad_hook(self._hook(i))
                      for i, p in enumerate(params)]
        self.pushes = 0

    # -- addresses ----------------------------------------------------------------------
    def _flag_area(self, r: int) -> int:
        return self.buf.bases[r]

    def _slot_addr(self, owner: int, elem_in_shard: int) -> int:
        return self.buf.bases[owner] + FLAG_BYTES + (self.rank * self.S + elem_in_shard) * 4

    def _push_range(self, a: int, b: int) -> None:
        """Copy flat_grad[a:b] into the owners' inbox slots (on the current stream)."""
        while a < b:
            owner = a // self.S
            end = min(b, (owner + 1) * self.S)
            ext().copy_to_address(self.flat_grad[a:end], self._slot_addr(owner, a - owner * self.S))
            self.pushes += 1
            a = end

    # -- per step -------------------------------------------------------------------------
    def arm(self) -> None:
        """The next backward is the step's last: push each gradient as soon as it is final."""
        self.armed = True
        self.pushed = [False] * len(self.ranges)

    def _hook(self, i: int):
        def hook(p):
            if not self.armed:
                return
            if self.pushed[i]:
                raise RuntimeError("a trainable tensor received two gradients in one backward; "
                                   "the overlapped reduce-scatter needs one per step")
            self.pushed[i] = True
            self.side.wait_stream(torch.cuda.current_stream(self.flat_grad.device))
            with torch.cuda.stream(self.side):
                self._push_range(*self.ranges[i])
        return hook

    def finish(self) -> torch.Tensor:
        """Complete the step's reduce-scatter; returns the device tensor holding the sum of
        squares of this rank's reduced shard."""
        cur = torch.cuda.current_stream(self.flat_grad.device)
        self.side.wait_stream(cur)
        self.epoch += 1
        with torch.cuda.stream(self.side):
            for i, done in enumerate(self.pushed if self.armed else [False] * len(self.ranges)):
                if not done:
                    self._push_range(*self.ranges[i])
            ext().grad_signal([self._flag_area(r) for r in range(self.world)], self.rank,
                              self.epoch)
        cur.wait_stream(self.side)
        self.sumsq.zero_()
        ext().grad_reduce(self.buf.bases[self.rank] + FLAG_BYTES, self._flag_area(self.rank),
                          self.world, self.epoch, self.shard_grad, self.sumsq, self.timeout_s)
        self.armed = False
        return self.sumsq

    def check(self) -> None:
        """Raise if a reduction gave up waiting for a peer (reads the device error word)."""
        check_device_error()

    def close(self) -> None:
        for h in self.hooks:
            h.remove()
        self.buf.close()
