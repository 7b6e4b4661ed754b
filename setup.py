"""Build the llmt native extensions in place (sm_100a only).

    python setup.py build_ext --inplace

Produces llmt/_C*.so (the release build) and llmt/_C_bounds*.so: the same sources compiled with
-DLLMT_DEBUG_BOUNDS=1, where every guarded global access checks its index range against the
extents of its launch, records the first violation and skips the access (a stand-in for a
memory sanitizer; selected at run time with LLMT_BOUNDS=1). Every .cu file under csrc/ is
compiled with -gencode arch=compute_100a,code=sm_100a; there is no other architecture.
LLMT_NO_BOUNDS_BUILD=1 skips the second module.
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
if os.environ.get("LLMT_PTXAS_VERBOSE"):
    NVCC += ["-Xptxas", "-v"]

sources = sorted(glob.glob(os.path.join("csrc", "**", "*.cu"), recursive=True)) + ["csrc/bindings.cpp"]


def bounds_sources():
    """One wrapper per source under build/bounds_src (distinct object paths for the second
    module); each includes the original file."""
    out = []
    for src in sources:
        dst = os.path.join("build", "bounds_src", src)
        os.makedirs(os.path.dirname(dst), exist_ok=True)
        text = f'#include "{os.path.join(ROOT, src)}"\n'
        if not os.path.exists(dst) or open(dst).read() != text:
            with open(dst, "w") as f:
                f.write(text)
        out.append(dst)
    return out


def ext(name, srcs, defines):
    return CUDAExtension(
        name=name,
        sources=srcs,
        include_dirs=[os.path.join(ROOT, "csrc")],
        extra_compile_args={"cxx": ["-O3", "-std=c++17"] + defines, "nvcc": NVCC + defines},
    )


modules = [ext("llmt._C", sources, [])]
if not os.environ.get("LLMT_NO_BOUNDS_BUILD"):
    modules.append(ext("llmt._C_bounds", bounds_sources(), ["-DLLMT_DEBUG_BOUNDS=1"]))

setup(
    name="llmt",
    packages=[],
    ext_modules=modules,
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
