"""Build recipe for the two in-tree native libraries of the ``ada_mla`` package.

* ``libmla_b200.so`` -- every CUDA kernel plus the C ABI of
  ``include/mla_b200.h``, compiled by nvcc for sm_100a only
  (``-gencode arch=compute_100a,code=sm_100a``).
* ``_ext/_ada_mla_ext.so`` -- the PyTorch extension (``csrc/mla_api.cpp``),
  which links ``libmla_b200.so`` and only calls its C ABI.

Both are built in-tree so they travel with the repository; nothing is
installed into site-packages and importing the package never compiles.
The reference JIT-builds its extension on every run through
``torch.utils.cpp_extension.load`` (mla.py:13-25) with sm_80/sm_89 flags.
"""
from __future__ import annotations

import glob
import os
import subprocess

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
PROJECT_DIR = os.path.dirname(PKG_DIR)                    # ada-mla_b200/
REPO_DIR = os.path.dirname(PROJECT_DIR)
CSRC_DIR = os.path.join(PROJECT_DIR, "csrc")
INCLUDE_DIR = os.path.join(REPO_DIR, "include")
LIB_PATH = os.path.join(PKG_DIR, "libmla_b200.so")
EXT_DIR = os.path.join(PKG_DIR, "_ext")
EXT_NAME = "_ada_mla_ext"
EXT_PATH = os.path.join(EXT_DIR, EXT_NAME + ".so")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
# Hidden visibility: only the MLA_B200_API entry points of include/mla_b200.h
# are exported (not the kernels' host stubs nor the static CUDA runtime).
NVCC_FLAGS = ARCH_FLAGS + ["-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
                           "-Xcompiler", "-Wall", "-Xcompiler", "-fvisibility=hidden"]


def _sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC_DIR, "*.cu")) +
                  glob.glob(os.path.join(CSRC_DIR, "*.cuh")) +
                  glob.glob(os.path.join(INCLUDE_DIR, "*.h")))


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.isfile(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = os.path.join(cuda_home, "bin", "nvcc")
    return path if os.path.isfile(path) else "nvcc"


def build_lib(force: bool = False, verbose: bool = False) -> str:
    """Compile csrc/mla_b200.cu (which includes every kernel) into LIB_PATH."""
    if not force and not _stale(LIB_PATH, _sources()):
        return LIB_PATH
    cmd = [nvcc(), *NVCC_FLAGS, "-I", INCLUDE_DIR, "-shared",
           "-Xlinker", "-soname=libmla_b200.so",
           "-o", LIB_PATH + ".tmp", os.path.join(CSRC_DIR, "mla_b200.cu")]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(LIB_PATH + ".tmp", LIB_PATH)
    return LIB_PATH


def build_ext(force: bool = False, verbose: bool = False) -> str:
    """Compile csrc/mla_api.cpp into the torch extension EXT_PATH."""
    import ctypes

    src = os.path.join(CSRC_DIR, "mla_api.cpp")
    deps = [src, LIB_PATH] + glob.glob(os.path.join(INCLUDE_DIR, "*.h"))
    if not force and not _stale(EXT_PATH, deps):
        return EXT_PATH
    from torch.utils import cpp_extension

    os.makedirs(EXT_DIR, exist_ok=True)
    ctypes.CDLL(LIB_PATH, mode=ctypes.RTLD_GLOBAL)
    cpp_extension.load(
        name=EXT_NAME,
        sources=[src],
        extra_include_paths=[INCLUDE_DIR],
        extra_cflags=["-O2"],
        extra_ldflags=[f"-L{PKG_DIR}", "-lmla_b200"],
        build_directory=EXT_DIR,
        with_cuda=True,
        verbose=verbose,
    )
    os.utime(EXT_PATH)
    return EXT_PATH


def build(force: bool = False, verbose: bool = False) -> None:
    build_lib(force=force, verbose=verbose)
    build_ext(force=force, verbose=verbose)


if __name__ == "__main__":
    import sys

    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB_PATH)
    print(EXT_PATH)
