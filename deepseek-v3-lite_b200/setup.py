"""Build the sm_100a kernel library in place: ``python setup.py build_ext --inplace``.

Produces ``ops/_dsv3_C.*.so`` inside this source tree.  Every CUDA source is
compiled for ``sm_100a`` only (tcgen05 / TMA need the architecture-specific
target); nothing here is portable to other GPUs by design.
"""
import os
from pathlib import Path

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = Path(__file__).resolve().parent
os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
os.environ.setdefault("MAX_JOBS", str(min(8, os.cpu_count() or 1)))

SOURCES = ["csrc/bindings.cpp", "csrc/status.cu", "csrc/gemm.cu", "csrc/elementwise.cu", "csrc/moe.cu",
           "csrc/attention.cu", "csrc/optim.cu", "csrc/comm.cu", "csrc/ep.cu", "csrc/dp.cu",
           "csrc/latent_decode_noalloc.cu"]

NVCC = ["-O3", "-lineinfo", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a",
        "--expt-relaxed-constexpr", "-Xptxas", "-v" if os.environ.get("DSV3_PTXAS_VERBOSE") else "-O3",
        "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_BFLOAT16_CONVERSIONS__"]
if os.environ.get("DSV3_CHECKS"):
    NVCC.append("-DDSV3_CHECKS=1")

setup(
    name="dsv3_b200_kernels",
    ext_modules=[CUDAExtension(
        name="ops._dsv3_C",
        sources=SOURCES,
        extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC},
    )],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
