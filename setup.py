"""Build the native parts of flodl_b200 in-tree.

Two extensions:

* ``flodl_b200._C``      hand-written sm_100a CUDA kernels (tcgen05 GEMM, flash
  attention, fused norms/losses/optimizers, peer-memory collectives) and their
  torch bindings. Compiled for ``sm_100a`` only.
* ``flodl_b200._native`` the C++ runtime that does not touch the GPU: ``.fdl``
  checkpoint IO, SHA-256/HMAC, graph topology compiler, ElChe cadence
  balancer, CPU averaging reducer and the batch prefetcher.

Usage: ``python setup.py build_ext --inplace -t /tmp/flodl_b200_build`` (``__graft_entry__.build()`` runs
exactly this).
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CppExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("flodl_b200", "csrc")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-diag-suppress", "177",
    "-DNDEBUG",
]
CXX_FLAGS = ["-O3", "-std=c++17", "-DNDEBUG", "-g0"]


def _shared_libstdcxx_dir():
    """Directory holding the SHARED libstdc++ link library.

    A toolchain whose private library directory only carries ``libstdc++.a``
    links a second, static copy of libstdc++ into each extension; that copy's
    iostream/locale state is never initialised, so formatting a number in an
    error message (``TORCH_CHECK(..., n)``) crashes. Putting the system
    directory first makes both extensions use the process-wide libstdc++.so.6
    that torch already loaded.
    """
    import subprocess

    for cxx in ("/usr/bin/g++", "g++", "c++"):
        try:
            out = subprocess.run([cxx, "-print-file-name=libstdc++.so"], capture_output=True,
                                 text=True, timeout=30).stdout.strip()
        except Exception:
            continue
        if os.path.isabs(out) and os.path.exists(out):
            return [os.path.dirname(out)]
    return []


LINK_DIRS = _shared_libstdcxx_dir()
LINK_FLAGS = [f"-L{d}" for d in LINK_DIRS]


def _sources(*patterns):
    out = []
    for p in patterns:
        out.extend(sorted(glob.glob(os.path.join(CSRC, p))))
    return out


ext_modules = [
    CUDAExtension(
        name="flodl_b200._C",
        sources=_sources("bind/*.cpp", "capi/*.cpp", "kernels/*.cu", "comm/*.cu"),
        include_dirs=[os.path.join(ROOT, CSRC)],
        extra_compile_args={"cxx": CXX_FLAGS, "nvcc": NVCC_FLAGS},
        extra_link_args=LINK_FLAGS,
    ),
    CppExtension(
        name="flodl_b200._native",
        sources=_sources("runtime/*.cpp"),
        include_dirs=[os.path.join(ROOT, CSRC)],
        extra_compile_args={"cxx": CXX_FLAGS},
        libraries=["z"],
        extra_link_args=LINK_FLAGS,
    ),
]

setup(
    name="flodl_b200",
    version="0.1.0",
    packages=["flodl_b200"],
    ext_modules=ext_modules,
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
