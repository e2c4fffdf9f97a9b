"""Scatter of per-rank Python payloads (a step's training samples) over the CPU control group,
with the array data sent as raw bytes.

``torch.distributed.scatter_object_list`` pickles every payload in-band: each numpy array is
copied into the pickle, the pickle is copied into a tensor, and every rank's tensor is padded
to the largest.  One rank's share of a 131k-token step (token ids, masks, log-probs and the
[T, L, K] routing ids) is about 21 MB, and rank 0 serialised all of them before any rank could
start: about 40 ms per rank on the host, so 0.3 s at eight ranks.  Here each payload is
pickled with protocol 5 and out-of-band buffers: the pickle holds only the object structure,
the arrays' bytes are laid out once (64-byte aligned) in one uint8 buffer per rank, and that
buffer goes to its rank with a point-to-point send.  The receiver rebuilds the objects with
their arrays as views of the received buffer (no further copy).
"""
from __future__ import annotations

import pickle
from typing import Any

import numpy as np
import torch
import torch.distributed as dist

_ALIGN = 64


def _align(n: int) -> int:
    return (n + _ALIGN - 1) // _ALIGN * _ALIGN


def pack(obj: Any) -> np.ndarray:
    """One uint8 buffer: [u64 meta length][meta pickle][structure pickle][array bytes...], with
    the structure and every array starting on a 64-byte boundary."""
    bufs: list[pickle.PickleBuffer] = []
    structure = pickle.dumps(obj, protocol=5, buffer_callback=bufs.append)
    raws = [b.raw() for b in bufs]
    sizes = [r.nbytes for r in raws]
    # meta: structure length and the buffers' sizes; its own length is fixed by a first pass
    meta = pickle.dumps((len(structure), sizes), protocol=5)
    head = _align(8 + len(meta))
    offsets, off = [], _align(head + len(structure))
    for n in sizes:
        offsets.append(off)
        off = _align(off + n)
    out = np.empty(off, dtype=np.uint8)
    out[:8] = np.frombuffer(len(meta).to_bytes(8, "little"), dtype=np.uint8)
    out[8:8 + len(meta)] = np.frombuffer(meta, dtype=np.uint8)
    out[head:head + len(structure)] = np.frombuffer(structure, dtype=np.uint8)
    for o, r in zip(offsets, raws):
        out[o:o + r.nbytes] = np.frombuffer(r, dtype=np.uint8)
    return out


def unpack(buf: np.ndarray) -> Any:
    """Inverse of ``pack``; arrays in the result are views of ``buf``."""
    mlen = int.from_bytes(buf[:8].tobytes(), "little")
    slen, sizes = pickle.loads(buf[8:8 + mlen].tobytes())
    head = _align(8 + mlen)
    structure = buf[head:head + slen]
    views, off = [], _align(head + slen)
    for n in sizes:
        views.append(buf[off:off + n])
        off = _align(off + n)
    return pickle.loads(structure, buffers=views)


def scatter(payloads: list | None, group=None, src: int = 0) -> Any:
    """Every rank of ``group`` calls this; rank ``src`` (a global rank) passes one payload per
    rank of the group (in group-rank order) and each rank gets its own back.  ``src``'s own
    payload is returned as it is."""
    world = dist.get_world_size(group)
    members = ([dist.get_global_rank(group, r) for r in range(world)] if group is not None
               else list(range(world)))
    rank = dist.get_rank()
    me = members.index(rank)
    if rank == src:
        if payloads is None or len(payloads) != world:
            raise ValueError(f"scatter needs {world} payloads on the source rank")
        packed = [None if g == src else pack(p) for g, p in zip(members, payloads)]
        sizes = torch.tensor([0 if b is None else b.nbytes for b in packed], dtype=torch.int64)
    else:
        sizes = torch.empty(world, dtype=torch.int64)
    dist.broadcast(sizes, src=src, group=group)
    if rank == src:
        works = [dist.isend(torch.from_numpy(packed[i]), dst=g, group=group)
                 for i, g in enumerate(members) if g != src]
        for w in works:
            w.wait()
        return payloads[members.index(src)]
    buf = torch.empty(int(sizes[me]), dtype=torch.uint8)
    dist.recv(buf, src=src, group=group)
    return unpack(buf.numpy())
