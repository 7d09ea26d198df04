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
import subprocess

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))


def _links_shared_libstdcxx(cxx: str) -> bool:
    """True if `cxx` finds a shared libstdc++ (it prints a bare name when it has none)."""
    try:
        out = subprocess.run([cxx, "-print-file-name=libstdc++.so"], capture_output=True, text=True,
                             timeout=30).stdout.strip()
    except (OSError, subprocess.SubprocessError):
        return False
    return os.path.isabs(out) and os.path.exists(out)


# A compiler that links libstdc++ statically gives each extension its own copy of the C++
# stream code next to the process's shared one; torch's error formatting (TORCH_CHECK
# with numbers) then crashes inside the extension instead of raising.  Prefer a compiler
# (and nvcc host compiler, via CC) that links the shared libstdc++.
if not _links_shared_libstdcxx(os.environ.get("CXX", "c++")):
    for var, name in (("CC", "gcc"), ("CXX", "g++")):
        for d in ("/usr/bin", "/usr/local/bin"):
            cand = os.path.join(d, name)
            if os.path.exists(cand) and (var == "CC" or _links_shared_libstdcxx(cand)):
                os.environ[var] = cand
                break
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
