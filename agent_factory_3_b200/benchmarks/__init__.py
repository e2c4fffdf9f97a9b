"""Kernel and end-to-end micro-benchmarks (CUDA-event timed; see ``kernels.py``)."""
