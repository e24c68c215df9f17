"""Build the native parts of gmm_b200 in-tree.

* ``gmm_b200/libgmm_sm100.so`` -- CUDA kernels + the C ABI of ``include/gmm_sm100.h``,
  compiled by nvcc for ``sm_100a`` only (``-gencode arch=compute_100a,code=sm_100a``).
* ``gmm_b200/_C.so`` -- the ``hopper_gmm_fwd::gmm`` torch operator (TORCH_LIBRARY,
  loaded with ``torch.ops.load_library``), linked against ``libgmm_sm100.so``.

Usage: ``python -m gmm_b200.build [--force]``.
"""

from __future__ import annotations

import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

LIB = os.path.join(PKG, "libgmm_sm100.so")
TORCH_OP = os.path.join(PKG, "_C.so")

KERNEL_SOURCES = [os.path.join(CSRC, f) for f in ("gmm_sm100.cu", "moe_sm100.cu")]
KERNEL_HEADERS = [os.path.join(CSRC, "sm100_ptx.cuh"), os.path.join(CSRC, "gmm_pair_kernel.cuh"),
                  os.path.join(CSRC, "gmm_vark_kernel.cuh"),
                  os.path.join(CSRC, "gmm_swap_kernel.cuh"),
                  os.path.join(INCLUDE, "gmm_sm100.h")]


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.check_call(cmd)


def build_kernels(force=False, verbose=True, extra=()):
    if force or _stale(LIB, KERNEL_SOURCES + KERNEL_HEADERS):
        _run([NVCC, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
              "-I", INCLUDE, *extra, "-o", LIB, *KERNEL_SOURCES], verbose)
    return LIB


def build_torch_op(force=False, verbose=True):
    src = os.path.join(CSRC, "torch_op.cpp")
    if not (force or _stale(TORCH_OP, [src, LIB, os.path.join(INCLUDE, "gmm_sm100.h")])):
        return TORCH_OP
    import torch
    from torch.utils import cpp_extension as ce
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    incs = []
    for p in ce.include_paths() + [os.path.join(CUDA_HOME, "include"), INCLUDE]:
        incs += ["-I", p]
    libdirs = []
    for p in ce.library_paths():
        libdirs += ["-L", p, f"-Wl,-rpath,{p}"]
    _run(["g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
          *incs, src, "-o", TORCH_OP, *libdirs, "-L", PKG, "-lgmm_sm100",
          "-Wl,-rpath,$ORIGIN", "-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch"], verbose)
    return TORCH_OP


def build_all(force=False, verbose=True):
    build_kernels(force, verbose)
    build_torch_op(force, verbose)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv)
