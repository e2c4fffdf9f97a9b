"""Sharded frozen base for data-parallel LoRA training (the role FSDP2 plays in the reference,
``examples/wordle/accelerate_config.yaml:1-13``, ``trainer/model_trainer.py:151-153``).

The reference wraps every decoder layer in FSDP2, so each rank stores 1/W of the weights and an
NCCL all-gather rebuilds a layer before its forward, its recompute and its backward.  On
B200 only the MXFP4 experts are worth sharding (64 of gpt-oss-120b's 65 GB; the bf16 attention
and embedding weights stay replicated), and the all-gather is not a separate collective:

* each rank keeps the experts [r*E/W, (r+1)*E/W) of every layer in one buffer of its own
  (``PeerMappedBuffer``: cudaMalloc + CUDA IPC, mapped by every rank of the node);
* when a layer needs its bf16 experts, one kernel (``mxfp4_dequant_gather``) reads each
  expert's packed e2m1 bytes and e8m0 scales straight from the owning rank's buffer over
  NVLink (plain loads) and writes the dequantised bf16 rows to this GPU's scratch -- the
  packed bytes (4.25 bits per weight) cross NVLink once and no packed copy is materialised;
* the frozen weights never change after set-up, so no flag or barrier guards the reads:
  the collective that exchanged the buffer handles is the only synchronisation needed.

On CPU (gloo, tests) the shards are gathered with ``all_gather`` instead, with the same
results.  Per rank the experts then take 1/W of their replicated size (gpt-oss-120b: 7.6 GB
instead of 61 GB at W = 8).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops import mxfp4
from ..ops._ext import ext


class ExpertShards:
    """Where one layer's experts live when they are sharded over the ranks of ``group``."""

    def __init__(self, group, world: int, rank: int, experts_per_rank: int, shapes: dict,
                 buffer=None, offsets: dict | None = None):
        self.group, self.world, self.rank = group, world, rank
        self.experts_per_rank = experts_per_rank
        self.shapes = shapes            # full shapes: {"gu_blocks": (E, N, G, 16), ...}
        self.buffer = buffer            # PeerMappedBuffer (CUDA) or None (CPU)
        self.offsets = offsets or {}
        self.ptr_tables: dict = {}
        if buffer is not None:
            dev = buffer.device
            for key, off in self.offsets.items():
                self.ptr_tables[key] = torch.tensor([b + off for b in buffer.bases],
                                                    dtype=torch.int64, device=dev)

    def dequantized(self, which: str, local_blocks: torch.Tensor, local_scales: torch.Tensor,
                    out: torch.Tensor | None) -> torch.Tensor:
        """bf16 [E, N, K] of the whole expert stack ``which`` ("gu" or "dn")."""
        if self.buffer is not None:
            ext().mxfp4_dequant_gather(self.ptr_tables[which + "_blocks"],
                                       self.ptr_tables[which + "_scales"],
                                       self.experts_per_rank, out)
            return out
        blocks = _all_gather(local_blocks, self.group, self.world)
        scales = _all_gather(local_scales, self.group, self.world)
        return mxfp4.dequantize(blocks, scales, out=out)

    def packed(self, which: str, local: torch.Tensor) -> torch.Tensor:
        """The full packed tensor ``which`` (e.g. "gu_blocks") gathered from every rank."""
        if self.buffer is None:
            return _all_gather(local, self.group, self.world)
        full = torch.empty(self.shapes[which], dtype=torch.uint8, device=local.device)
        chunk = full.view(self.world, -1)
        off = self.offsets[which]
        for r, base in enumerate(self.buffer.bases):
            ext().copy_from_address(base + off, chunk[r])
        return full


def _all_gather(t: torch.Tensor, group, world: int) -> torch.Tensor:
    parts = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(parts, t.contiguous(), group=group)
    return torch.cat(parts, 0)


_KEYS = (("gu_blocks", "gate_up_blocks"), ("gu_scales", "gate_up_scales"),
         ("dn_blocks", "down_blocks"), ("dn_scales", "down_scales"))


def shard_expert_weights(model, group=None) -> list[ExpertShards]:
    """Keep only this rank's experts of every MoE layer; the others are read from their owners
    (see the module docstring).  Every rank of ``group`` must call this with the same model
    (same weights).  Returns the per-layer shard descriptors (also attached to the layers)."""
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    out = []
    for layer in model.layers:
        mlp = layer.mlp
        E = mlp.gate_up_blocks.shape[0]
        if E % world:
            raise ValueError(f"{E} experts cannot be split evenly over {world} ranks")
        epr = E // world
        sl = slice(rank * epr, (rank + 1) * epr)
        shapes = {k: tuple(getattr(mlp, attr).shape) for k, attr in _KEYS}
        dev = mlp.gate_up_blocks.device
        if dev.type == "cuda":
            from .symm import PeerMappedBuffer
            offs, total = {}, 0
            for k, attr in _KEYS:
                offs[k] = total
                n = getattr(mlp, attr)[sl].numel()
                total += (n + 255) // 256 * 256
            buf = PeerMappedBuffer(total, group, dev)
            for k, attr in _KEYS:
                src = getattr(mlp, attr)[sl]
                view = buf.local[offs[k]:offs[k] + src.numel()].view(src.shape)
                view.copy_(src)
                setattr(mlp, attr, view)       # replaces the full registered buffer
            torch.cuda.synchronize(dev)
            dist.barrier(group=group)          # every shard is written before anyone reads
            sh = ExpertShards(group, world, rank, epr, shapes, buf, offs)
        else:
            for _, attr in _KEYS:
                setattr(mlp, attr, getattr(mlp, attr)[sl].clone())
            sh = ExpertShards(group, world, rank, epr, shapes)
        mlp.expert_shards = sh
        out.append(sh)
    if torch.cuda.is_available():
        torch.cuda.empty_cache()
    return out
