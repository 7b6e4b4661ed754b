"""Build the llmt native extension in place (sm_100a only).

    python setup.py build_ext --inplace

Produces llmt/_C*.so. Every .cu file under csrc/ is compiled with
-gencode arch=compute_100a,code=sm_100a; there is no other architecture.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC = ARCH + ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr", "-DNDEBUG",
               "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
               "-U__CUDA_NO_BFLOAT16_CONVERSIONS__", "-U__CUDA_NO_HALF2_OPERATORS__"]
if os.environ.get("LLMT_DEBUG_BOUNDS"):
    NVCC += ["-DLLMT_DEBUG_BOUNDS=1"]
if os.environ.get("LLMT_PTXAS_VERBOSE"):
    NVCC += ["-Xptxas", "-v"]

sources = sorted(glob.glob(os.path.join("csrc", "**", "*.cu"), recursive=True)) + ["csrc/bindings.cpp"]

setup(
    name="llmt",
    packages=[],
    ext_modules=[CUDAExtension(
        name="llmt._C",
        sources=sources,
        include_dirs=[os.path.join(ROOT, "csrc")],
        extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC},
    )],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
