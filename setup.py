"""Build the native parts of revealaiccl_b200 in-tree.

    python setup.py build_ext --inplace

produces
  revealaiccl_b200/_kernels*.so  sm_100a CUDA kernels (tcgen05/TMEM/TMA, peer stores)
  revealaiccl_b200/_host*.so     host C++ runtime (event bridge, compiled scheduler core,
                                 peer channel handle exchange)
Every CUDA source is compiled for sm_100a only.
"""

import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
INC = [os.path.join(ROOT, "csrc", "include")]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC = ARCH + ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xptxas", "-v"]
CXX = ["-O3", "-std=c++17"]


def _sources(sub, exts):
    folder = os.path.join("csrc", sub)
    return sorted(os.path.join(folder, f) for f in os.listdir(folder) if f.endswith(exts))


ext_modules = [
    CUDAExtension(
        "revealaiccl_b200._kernels",
        sources=_sources("kernels", (".cu", ".cpp")),
        include_dirs=INC,
        extra_compile_args={"cxx": CXX, "nvcc": NVCC},
    ),
]
if os.path.isdir(os.path.join(ROOT, "csrc", "host")) and _sources("host", (".cpp",)):
    ext_modules.append(
        CUDAExtension(
            "revealaiccl_b200._host",
            sources=_sources("host", (".cpp", ".cu")),
            include_dirs=INC,
            extra_compile_args={"cxx": CXX + ["-pthread"], "nvcc": NVCC},
        )
    )

setup(
    name="revealaiccl_b200",
    version="0.1.0",
    packages=["revealaiccl_b200"],
    ext_modules=ext_modules,
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
