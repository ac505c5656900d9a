"""Build ``libm3gemv.so`` in-tree with nvcc for sm_100a.

``python -m m3_avm_b200.build_lib`` (or ``build()``) compiles every ``.cu``
under ``csrc/`` into ``m3_avm_b200/libm3gemv.so``.  nvcc cross-compiles, so
this runs on a machine without a GPU.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
LIB = os.path.join(HERE, "libm3gemv.so")
E2E_SRC = os.path.join(HERE, "e2e_timing.c")
E2E_BIN = os.path.join(HERE, "m3g_e2e_timing")  # C timing of the host-buffer call (bench.py's e2e figure)

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps() -> list[str]:
    return sources() + sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))) + [
        os.path.join(INCLUDE, "m3gemv.h")
    ]


def up_to_date() -> bool:
    if not os.path.exists(LIB) or not os.path.exists(E2E_BIN):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(p) <= t for p in _deps())


def build(force: bool = False, verbose_ptxas: bool = False) -> str:
    """Compile the library if any source is newer than it; return its path."""
    if not force and up_to_date():
        return LIB
    gcc = shutil.which("g++") or "/usr/bin/g++"
    cmd = [
        nvcc_path(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "--shared", "-Xcompiler", "-fPIC",
        "-Xcompiler", "-fvisibility=hidden", "-ccbin", gcc, "-I", INCLUDE, "-I", CSRC,
        "-DM3G_BUILD_LIB", "-o", LIB + ".tmp", *sources(), "-lnccl",
    ]
    if verbose_ptxas:
        cmd[1:1] = ["-Xptxas", "-v"]
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    build_e2e(force=True)
    return LIB


def build_e2e(force: bool = False) -> str:
    """The C program that times m3g_offload_matvec against libm3gemv.so."""
    if not force and os.path.exists(E2E_BIN) and os.path.getmtime(E2E_BIN) >= max(
            os.path.getmtime(E2E_SRC), os.path.getmtime(LIB)):
        return E2E_BIN
    gcc = shutil.which("gcc") or "/usr/bin/gcc"
    subprocess.run([gcc, "-O2", "-std=c11", "-Wall", "-I", INCLUDE, "-o", E2E_BIN + ".tmp", E2E_SRC, "-L", HERE,
                    "-lm3gemv", "-Wl,-rpath,$ORIGIN"], check=True)
    os.replace(E2E_BIN + ".tmp", E2E_BIN)
    return E2E_BIN


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose_ptxas="-v" in sys.argv)
    print(LIB)
