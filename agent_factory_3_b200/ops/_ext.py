"""Loader of the in-tree sm_100a extension (``agent_factory_3_b200/_C*.so``).

On a machine with a CUDA device the extension is mandatory: operators called with CUDA
tensors raise instead of silently falling back to PyTorch.  On CPU-only machines the
operators use their PyTorch reference implementations.
"""
from __future__ import annotations

import importlib
import os

import torch

_EXT = None
_ERR: Exception | None = None

# Kernel launches issued by each extension entry point (for the launch counter below).
_LAUNCHES_PER_CALL = {"moe_group": 4, "attn_bwd": 3, "decode_attention": 2, "device_error": 0}
_launch_count = 0


_NVTX = os.environ.get("AF3_NVTX") == "1"


class _CountingExt:
    """Proxy of the extension module that counts the kernels its entry points launch.  With
    AF3_NVTX=1 every entry point also runs inside an NVTX range named ``af3.<entry point>``,
    so a timeline profiler shows which native op issued each kernel."""

    def __init__(self, mod):
        self._mod = mod

    def __getattr__(self, name):
        fn = getattr(self._mod, name)
        if not callable(fn):
            return fn
        n = _LAUNCHES_PER_CALL.get(name, 1)

        if _NVTX:
            def call(*a, **k):
                global _launch_count
                _launch_count += n
                torch.cuda.nvtx.range_push(f"af3.{name}")
                try:
                    return fn(*a, **k)
                finally:
                    torch.cuda.nvtx.range_pop()
            return call

        def call(*a, **k):
            global _launch_count
            _launch_count += n
            return fn(*a, **k)

        return call


def launch_count() -> int:
    """Number of this package's kernels launched so far in this process."""
    return _launch_count


def ext():
    """Return the compiled extension module, importing it on first use."""
    global _EXT, _ERR
    if _EXT is not None:
        return _EXT
    if _ERR is not None:
        raise RuntimeError(
            "agent_factory_3_b200._C is not available; build it with "
            "`python setup.py build_ext --inplace`"
        ) from _ERR
    try:
        _EXT = _CountingExt(importlib.import_module("agent_factory_3_b200._C"))
    except Exception as e:  # pragma: no cover - exercised on machines without the build
        _ERR = e
        raise RuntimeError(
            "agent_factory_3_b200._C is not available; build it with "
            "`python setup.py build_ext --inplace`"
        ) from e
    return _EXT


def available() -> bool:
    try:
        ext()
        return True
    except RuntimeError:
        return False


def use_cuda_kernels(*tensors: torch.Tensor) -> bool:
    """True when every tensor is on a CUDA device (the extension must then be present)."""
    if not tensors or not all(t.is_cuda for t in tensors if t is not None):
        return False
    if os.environ.get("AF3_FORCE_TORCH_REFERENCE") == "1":
        return False
    ext()  # raise loudly if missing
    return True


def check_device_error() -> None:
    """Raise if a bounded wait inside one of our kernels expired since the last check."""
    code = ext().device_error()
    if code != 0:
        raise RuntimeError(f"agent_factory_3_b200 kernel reported error code {code}")
