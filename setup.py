"""Build grappa_b200's native extensions in place.

    python setup.py build_ext --inplace      (no -j: the two extensions share one ninja build dir)

Two modules are built:
  grappa_b200/_C      host engine (C++17 + OpenMP, pybind11; no CUDA)
  grappa_b200/_cuda   sm_100a kernels (nvcc -gencode arch=compute_100a,code=sm_100a)
                      with their torch bindings
"""
import glob
import os

import pybind11
from setuptools import Extension, setup

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("grappa_b200", "csrc")
INC = [os.path.join(HERE, CSRC, "include")]

os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")

# The compiler driver of this image has no libgomp.spec next to it; the OpenMP
# runtime is linked explicitly from the system gcc.
GOMP_DIR = "/usr/lib/gcc/x86_64-linux-gnu/13"

host_ext = Extension(
    "grappa_b200._C",
    sources=sorted(glob.glob(os.path.join(CSRC, "host", "*.cc"))),
    include_dirs=INC + [pybind11.get_include()],
    extra_compile_args=["-O3", "-std=c++17", "-fopenmp", "-fvisibility=hidden", "-Wall",
                        "-Wno-sign-compare", "-Wno-unused-variable", "-Wno-unknown-pragmas"],
    extra_link_args=[f"-L{GOMP_DIR}", "-lgomp"],
    language="c++",
)

ext_modules = [host_ext]
cmdclass = {}

if os.environ.get("GRAPPA_SKIP_CUDA", "0") != "1":
    from torch.utils.cpp_extension import BuildExtension, CUDAExtension

    NVCC_FLAGS = [
        "-O3", "-std=c++17", "-lineinfo",
        "-gencode", "arch=compute_100a,code=sm_100a",
        "--expt-relaxed-constexpr", "-DNDEBUG",
    ]
    if os.environ.get("GRAPPA_PTXAS_V"):
        NVCC_FLAGS += ["-Xptxas", "-v"]
    cuda_ext = CUDAExtension(
        "grappa_b200._cuda",
        sources=sorted(glob.glob(os.path.join(CSRC, "cuda", "*.cu")))
        + sorted(glob.glob(os.path.join(CSRC, "cuda", "*.cpp"))),
        include_dirs=INC,
        extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
    )
    ext_modules.append(cuda_ext)
    cmdclass["build_ext"] = BuildExtension.with_options(use_ninja=True)

setup(
    name="grappa_b200",
    version="0.1.0",
    packages=["grappa_b200", "t10n"],
    ext_modules=ext_modules,
    cmdclass=cmdclass,
)
