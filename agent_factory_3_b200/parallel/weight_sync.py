"""Direct trainer -> rollout-engine weight sync through GPU memory.

The reference writes the adapter (or merged weights) to a shared filesystem and asks sglang to
reload it over HTTP (trainer/sglang_controller.py, rl_flow.py:949-954).  When the trainer and
the engine sit on one NVLink / NVSwitch box, the engine instead exports a flat bf16 staging
buffer by CUDA IPC; the trainer maps it and one kernel (``peer_cast_copy``) casts its fp32 LoRA
tensors to bf16 while storing them straight into the engine GPU's memory.  The engine then
applies the staged tensors to its LoRA parameters at a safe point between steps.

    # engine process
    stage = StagingBuffer.for_tensors(engine_lora_shapes, device)
    handle = stage.export()                     # picklable; send to the trainer
    # trainer process
    writer = PeerWriter(handle)
    writer.write(trainer_lora_tensors)          # one kernel over NVLink; returns when landed
    # engine: engine.control("apply_staged_lora", name, stage.tensors())
"""
from __future__ import annotations

import pickle
from dataclasses import dataclass

import torch

from ..ops._ext import ext, use_cuda_kernels


@dataclass
class LayoutEntry:
    name: str
    offset: int          # element offset in the flat buffer (multiple of 8)
    shape: tuple


def _align8(n: int) -> int:
    return (n + 7) // 8 * 8


class StagingBuffer:
    """Receiver side: one flat bf16 buffer holding every synced tensor at an aligned offset.
    On a GPU the buffer is its own ``cudaMalloc`` so its CUDA IPC handle covers exactly it."""

    def __init__(self, layout: list[LayoutEntry], numel: int, device, flat: torch.Tensor | None = None):
        self.layout = layout
        self.device = torch.device(device)
        self._handle = None
        if flat is None and self.device.type == "cuda" and use_cuda_kernels(torch.empty(0, device=self.device)):
            raw, self._handle = ext().symm_alloc(numel * 2, self.device.index)
            flat = raw.view(torch.bfloat16)
        self.flat = flat if flat is not None else torch.zeros(numel, dtype=torch.bfloat16, device=device)
        self.version = 0

    @classmethod
    def for_tensors(cls, shapes: dict[str, tuple], device) -> "StagingBuffer":
        layout, off = [], 0
        for name, shape in shapes.items():
            n = 1
            for d in shape:
                n *= int(d)
            layout.append(LayoutEntry(name, off, tuple(int(d) for d in shape)))
            off += _align8(n)
        return cls(layout, max(off, 8), device)

    def tensors(self) -> dict[str, torch.Tensor]:
        out = {}
        for e in self.layout:
            n = 1
            for d in e.shape:
                n *= d
            out[e.name] = self.flat[e.offset:e.offset + n].view(e.shape)
        return out

    def export(self) -> bytes:
        """Picklable description (CUDA IPC handle of the buffer + layout) for another process
        on the same machine."""
        if self._handle is None:
            raise RuntimeError("only a GPU staging buffer can be exported")
        return pickle.dumps({"handle": bytes(self._handle),
                             "layout": [(e.name, e.offset, e.shape) for e in self.layout],
                             "numel": self.flat.numel()})


class PeerWriter:
    """Sender side: maps a staging buffer exported by another process (or wraps a local one)
    and writes tensors into it with the fused cast + NVLink-store kernel.  The mapping is opened
    on ``device`` (default: the current CUDA device), with peer access enabled for it, so the
    writing kernel must run there."""

    def __init__(self, exported: bytes | StagingBuffer, device=None):
        self._opened = None
        if isinstance(exported, StagingBuffer):
            self.local = exported.flat
            self.dst_ptr, self.dst_numel = exported.flat.data_ptr(), exported.flat.numel()
            self.layout = exported.layout
            self.device = exported.flat.device
        else:
            d = pickle.loads(exported)
            self.local = None
            self.device = torch.device(device) if device is not None else \
                torch.device("cuda", torch.cuda.current_device())
            with torch.cuda.device(self.device):
                self._opened = ext().ipc_open(d["handle"])
            self.dst_ptr, self.dst_numel = self._opened, int(d["numel"])
            self.layout = [LayoutEntry(n, o, tuple(s)) for n, o, s in d["layout"]]
        self.offsets = {e.name: e.offset for e in self.layout}
        self.shapes = {e.name: e.shape for e in self.layout}
        self.bytes_written = 0

    def write(self, tensors: dict[str, torch.Tensor], stream_sync: bool = True) -> int:
        """Cast and store ``tensors`` (names of the layout) into the staging buffer; with
        ``stream_sync`` returns once the data has landed in the destination GPU's memory."""
        names = [n for n in tensors if n in self.offsets]
        missing = set(tensors) - set(names)
        if missing:
            raise KeyError(f"tensors not in the staging layout: {sorted(missing)[:5]}")
        srcs = [tensors[n].detach().contiguous() for n in names]
        for n, t in zip(names, srcs):
            if tuple(t.shape) != self.shapes[n]:
                raise ValueError(f"{n}: shape {tuple(t.shape)} != staged {self.shapes[n]}")
        offs = [self.offsets[n] for n in names]
        on_gpu = bool(srcs) and srcs[0].is_cuda and use_cuda_kernels(srcs[0])
        if on_gpu and all(t.numel() % 8 == 0 for t in srcs):
            if self._opened is not None and srcs[0].device != self.device:
                raise ValueError(f"sources on {srcs[0].device}, mapping opened on {self.device}")
            with torch.cuda.device(srcs[0].device):
                if self._opened is None and self.device != srcs[0].device:
                    ext().enable_peer_access(self.device.index)   # same-process peer buffer
                ext().peer_cast_copy(self.dst_ptr, self.dst_numel,
                                     [t if t.dtype in (torch.float32, torch.bfloat16)
                                      else t.float() for t in srcs], offs)
                if stream_sync:
                    torch.cuda.current_stream().synchronize()
        elif self.local is not None:
            for t, o in zip(srcs, offs):
                self.local[o:o + t.numel()].copy_(t.reshape(-1).to(torch.bfloat16))
        else:
            raise RuntimeError("remote staging buffers need the CUDA kernel path "
                               "(tensor sizes must be multiples of 8)")
        n_bytes = sum(t.numel() * 2 for t in srcs)
        self.bytes_written += n_bytes
        return n_bytes

    def close(self) -> None:
        if self._opened is not None:
            ext().ipc_close(self._opened)
            self._opened = None
