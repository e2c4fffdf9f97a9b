"""Buffers that every rank of a process group has mapped (CUDA IPC over NVLink / NVSwitch).

Each rank allocates one buffer with its own ``cudaMalloc`` and shares the IPC handle with the
group (one ``all_gather_object``); every rank then opens the peers' handles, so a kernel on any
rank can load from or store to any rank's buffer by plain device addresses.  Layout of a
buffer: a 256-byte flag area (one uint32 arrival epoch per rank) followed by ``sets``
equally-sized data sets that alternate between successive collective calls.

The reference has no such layer: its rollout engine (sglang) reduces with NCCL or its own
custom all-reduce, and its trainer uses NCCL only.  Only plain peer mappings are made (no NVLS
switch-memory binding), so a rank that exits cannot fault the others through such a binding.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops._ext import ext

FLAG_BYTES = 256


class PeerMappedBuffer:
    """``nbytes`` of device memory on this rank, mapped by every other rank of ``group``.

    ``local`` is this rank's buffer (uint8 tensor); ``bases[j]`` is rank j's buffer as a
    device address valid on this rank (its own for j == rank).  Used for data that never
    changes after set-up (sharded frozen weights), so readers need no synchronisation beyond
    the collective that exchanged the handles."""

    def __init__(self, nbytes: int, group=None, device: torch.device | None = None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > 8:
            raise ValueError("peer mapping supports at most 8 ranks (one NVLink domain)")
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.local, handle = ext().symm_alloc(int(nbytes), self.device.index)
        handles: list = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self._opened: list[int] = []
        self.bases: list[int] = []
        with torch.cuda.device(self.device):
            for j, h in enumerate(handles):
                if j == self.rank:
                    self.bases.append(self.local.data_ptr())
                else:
                    p = ext().ipc_open(h)
                    self._opened.append(p)
                    self.bases.append(p)

    def close(self) -> None:
        for p in self._opened:
            try:
                ext().ipc_close(p)
            except Exception:  # noqa: BLE001 - unmapping at exit is best effort
                pass
        self._opened.clear()


class SymmetricWorkspace:
    def __init__(self, set_bytes: int, group=None, device: torch.device | None = None,
                 sets: int = 2):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > 8:
            raise ValueError("SymmetricWorkspace supports at most 8 ranks (one NVLink domain)")
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.set_bytes = (int(set_bytes) + 255) // 256 * 256
        self.sets = sets
        total = FLAG_BYTES + sets * self.set_bytes
        self.local, handle = ext().symm_alloc(total, self.device.index)
        handles: list = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self._opened: list[int] = []
        self.bases: list[int] = []
        with torch.cuda.device(self.device):
            for j, h in enumerate(handles):
                if j == self.rank:
                    self.bases.append(self.local.data_ptr())
                else:
                    p = ext().ipc_open(h)
                    self._opened.append(p)
                    self.bases.append(p)
        self.epoch = 0

    # addresses -------------------------------------------------------------------------
    def flag_ptrs(self) -> list[int]:
        return list(self.bases)

    def set_ptrs(self, s: int) -> list[int]:
        return [b + FLAG_BYTES + s * self.set_bytes for b in self.bases]

    def local_set(self, s: int, shape, dtype=torch.bfloat16) -> torch.Tensor:
        n = 1
        for d in shape:
            n *= int(d)
        nbytes = n * torch.empty(0, dtype=dtype).element_size()
        if nbytes > self.set_bytes:
            raise ValueError(f"{nbytes} bytes do not fit a {self.set_bytes}-byte set")
        off = FLAG_BYTES + s * self.set_bytes
        return self.local[off:off + nbytes].view(dtype).view(*shape)

    def close(self) -> None:
        for p in self._opened:
            try:
                ext().ipc_close(p)
            except Exception:
                pass
        self._opened.clear()
