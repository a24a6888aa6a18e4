"""Builds the sm_100a extension in-tree: ``python setup.py build_ext --inplace``.

Only Blackwell (sm_100a) code is generated: the ``-gencode`` flags below are the only arch
flags (torch adds none of its own when the user passes a ``-gencode``).
"""
import os

from setuptools import find_packages, setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("micro_engram_fork_b200", "csrc")

NVCC = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
]
if os.environ.get("ME_BOUNDS_CHECK") == "1":
    NVCC.append("-DME_BOUNDS_CHECK")
CXX = ["-O3", "-std=c++17"]

SOURCES = [os.path.join(CSRC, f) for f in (
    "bindings.cpp", "symm.cpp", "engram.cu", "norm.cu", "ce.cu", "attention.cu", "attention_tc.cu", "gemm.cu", "gemm_fused.cu", "gemm_nf4.cu",
    "p2p.cu", "nf4.cu",
)]

setup(
    name="micro_engram_fork_b200",
    version="0.1.0",
    packages=find_packages(include=["micro_engram*", "micro_engram_fork_b200*", "micro_engram_vllm*"]),
    ext_modules=[CUDAExtension(
        name="micro_engram_fork_b200._C",
        sources=SOURCES,
        include_dirs=[os.path.join(HERE, CSRC)],
        extra_compile_args={"cxx": CXX, "nvcc": NVCC},
    )],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
    entry_points={"vllm.general_plugins": ["micro_engram = micro_engram_vllm:register"]},
)
