"""Builds the sm_100a extension in place: ``python setup.py build_ext --inplace``.

The product is ``nanospec_b200/_C*.so`` inside the source tree (it is git-ignored
but travels with the tree to GPU machines). Architecture flags are passed
explicitly, so torch's own arch list does not matter.
"""

import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
os.environ.setdefault("MAX_JOBS", str(min(8, os.cpu_count() or 4)))

sources = sorted(glob.glob(os.path.join("csrc", "*.cu"))) + ["csrc/bindings.cpp"]
nvcc = [
    "-O3", "-std=c++17", "-lineinfo",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "--expt-relaxed-constexpr", "-Xptxas=-v" if os.environ.get("NS_PTXAS_VERBOSE") else "-Xptxas=-O3",
    "-DNDEBUG", "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT162_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
]
setup(
    name="nanospec_b200",
    packages=[],
    ext_modules=[
        CUDAExtension(
            "nanospec_b200._C",
            sources,
            include_dirs=[os.path.join(ROOT, "csrc", "include")],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": nvcc},
            libraries=["cuda"],
            library_dirs=["/usr/local/cuda/lib64/stubs"],
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
