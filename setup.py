"""Builds the sm_100a extension in-tree:  python setup.py build_ext --inplace

Every .cu file is compiled for sm_100a only (-gencode arch=compute_100a,code=sm_100a); the extension lands in
nanovllm_b200/_C*.so next to the Python package so it travels with the source tree.  The host-only helpers
(csrc/host, plain C++) build into nanovllm_b200/_host*.so.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CppExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "nanovllm_b200", "csrc")
sources = sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + [os.path.join(CSRC, "bindings.cpp")]
sources = [os.path.relpath(s, HERE) for s in sources]

nvcc_flags = [
    "-O3",
    "-std=c++17",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "--use_fast_math",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_OPERATORS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
    "--expt-relaxed-constexpr",
]
if os.environ.get("NANOVLLM_PTXAS_VERBOSE"):
    nvcc_flags.append("-Xptxas=-v")

setup(
    name="nanovllm_b200",
    version="0.1.0",
    packages=["nanovllm_b200"],
    ext_modules=[
        CUDAExtension(
            name="nanovllm_b200._C",
            sources=sources,
            include_dirs=[CSRC],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": nvcc_flags},
        ),
        # host-only runtime helpers (tokenizer core): plain C++, no CUDA
        CppExtension(
            name="nanovllm_b200._host",
            sources=[os.path.relpath(os.path.join(CSRC, "host", "bpe.cpp"), HERE)],
            extra_compile_args=["-O3", "-std=c++17"],
        ),
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
