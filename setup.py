"""Build the sm_100a kernel library in-tree: ``python setup.py build_ext --inplace``.

Produces ``titans_pytorch_b200/_C.*.so``.  The architecture flags are passed
explicitly (``-gencode arch=compute_100a,code=sm_100a``), so torch's own arch
list is not used.
"""

import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("titans_pytorch_b200", "csrc")

sources = sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + sorted(glob.glob(os.path.join(CSRC, "*.cpp")))

nvcc_flags = [
    "-O3",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_OPERATORS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
]
if os.environ.get("TITANS_PTXAS_VERBOSE") == "1":
    nvcc_flags.append("-Xptxas=-v")

setup(
    name="titans_pytorch_b200",
    version="0.1.0",
    packages=["titans_pytorch_b200"],
    ext_modules=[
        CUDAExtension(
            name="titans_pytorch_b200._C",
            sources=sources,
            include_dirs=[os.path.join(HERE, CSRC)],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": nvcc_flags},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
