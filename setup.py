"""Build the sm_100a CUDA extension in-tree: ``python setup.py build_ext --inplace``.

Produces ``shift_b200/_C*.so`` (kernels) next to the Python sources.  Only
sm_100a code is generated (``-gencode arch=compute_100a,code=sm_100a``).
The C++ control plane (lighthouse daemon and its client library) is built by
``shift_b200/ft/native_build.py`` with plain g++.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("shift_b200", "csrc")

cuda_flags = [
    "-O3",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-v",
]
if os.environ.get("SHIFT_DEBUG_BOUNDS"):
    cuda_flags.append("-DSHIFT_DEBUG_BOUNDS=1")

sources = sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + [os.path.join(CSRC, "bindings.cpp")]

setup(
    name="shift_b200",
    ext_modules=[
        CUDAExtension(
            name="shift_b200._C",
            sources=sources,
            include_dirs=[os.path.join(ROOT, CSRC)],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": cuda_flags},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
