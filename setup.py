"""Build of the sm_100a CUDA extension, in place:  python setup.py build_ext --inplace

Every .cu/.cpp file under agent_factory_3_b200/csrc is compiled for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``); torch's own arch list is bypassed.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("agent_factory_3_b200", "csrc")

sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))

nvcc_flags = [
    "-O3",
    "-std=c++17",
    "-gencode=arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT162_OPERATORS__",
    "-Xptxas=-warn-spills",
]
if os.environ.get("AF3_PTXAS_VERBOSE"):
    nvcc_flags.append("-Xptxas=-v")

os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")

setup(
    name="agent_factory_3_b200",
    version="0.1.0",
    packages=[],
    ext_modules=[
        CUDAExtension(
            name="agent_factory_3_b200._C",
            sources=sources,
            include_dirs=[os.path.join(HERE, CSRC)],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": nvcc_flags},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
