"""Build the zstep_b200 native components in-tree.

    python setup.py build_ext --inplace

produces
  * zstep_b200/_C*.so      -- sm_100a kernels (tcgen05 / TMA) + torch bindings
  * zstep_b200/_master*.so -- the C++ control plane (wire ABI, SHM transport, KV block
                              pool, prefix cache, scheduler, tokenizer, HTTP server) as a
                              Python module, used by tests and by the `zstep` launcher.
The stand-alone `zstep` executable is built by zstep_b200/build_native.py.
"""

import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
KDIR = os.path.join("csrc", "kernels")
MDIR = os.path.join("csrc", "master")

CUDA_FLAGS = [
    "-gencode=arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-O3",
    "-std=c++17",
    "--expt-relaxed-constexpr",
]

kernel_sources = [os.path.join(KDIR, f) for f in sorted(os.listdir(os.path.join(ROOT, KDIR)))
                  if f.endswith(".cu") or f == "bindings.cpp"]

ext_modules = [
    CUDAExtension(
        name="zstep_b200._C",
        sources=kernel_sources,
        include_dirs=[os.path.join(ROOT, KDIR)],
        extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": CUDA_FLAGS},
    ),
]

master_sources = sorted(
    os.path.join(MDIR, f) for f in os.listdir(os.path.join(ROOT, MDIR))
    if f.endswith(".cc") and not f.startswith("main_")
) if os.path.isdir(os.path.join(ROOT, MDIR)) else []

if master_sources:
    import pybind11
    from setuptools import Extension

    ext_modules.append(
        Extension(
            name="zstep_b200._master",
            sources=master_sources,
            include_dirs=[os.path.join(ROOT, MDIR), pybind11.get_include()],
            extra_compile_args=["-O2", "-std=c++17", "-fvisibility=hidden", "-Wall"],
            libraries=["pthread"],
            language="c++",
        )
    )

setup(
    name="zstep_b200",
    version="0.1.0",
    packages=["zstep_b200"],
    ext_modules=ext_modules,
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
