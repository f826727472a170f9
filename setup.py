"""Builds the sm_100a extension in place: `python setup.py build_ext --inplace -j 8`.

The kernels (.cu) include no torch headers, so they compile in seconds; only bindings.cpp pulls in torch.  The
explicit -gencode flag makes torch's extension builder skip its own architecture list: the binary holds sm_100a
code only (tcgen05 instructions do not exist on any other architecture).
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("inference_optimizations_b200", "csrc")
NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-lineinfo",
              "--expt-relaxed-constexpr", "-Xptxas", "-v" if os.environ.get("IOB_PTXAS_VERBOSE") else "-O3"]

sources = sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + [os.path.join(CSRC, "bindings.cpp")]

setup(
    name="inference_optimizations_b200",
    version="0.1.0",
    packages=[],
    ext_modules=[
        CUDAExtension(
            name="inference_optimizations_b200._C",
            sources=sources,
            include_dirs=[os.path.join(HERE, CSRC)],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS + os.environ.get("IOB_EXTRA_NVCC", "").split()},
            libraries=["cuda"],
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
