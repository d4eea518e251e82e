"""Build recipe for libztcp_b200.so (sm_100a).

Compiles the CUDA and host C++ sources in ``vlx-tee_b200/csrc`` with nvcc into
``vlx-tee_b200/ztcp_b200/libztcp_b200.so``, in-tree, so the built library
travels with the repository to GPU machines.  nvcc cross-compiles for sm_100a
without a GPU present.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(os.path.dirname(PKG_DIR), "csrc")
INCLUDE = os.path.join(os.path.dirname(os.path.dirname(PKG_DIR)), "include")
LIB_PATH = os.path.join(PKG_DIR, "libztcp_b200.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
]


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))


def _inputs() -> list[str]:
    return sources() + sorted(glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh"))) + [
        os.path.join(INCLUDE, "ztcp_b200.h"), os.path.join(INCLUDE, "ztcp_ledger.h"),
        os.path.join(INCLUDE, "ztcp_measure.h")
    ]


def up_to_date() -> bool:
    if not os.path.isfile(LIB_PATH):
        return False
    t = os.path.getmtime(LIB_PATH)
    return all(os.path.getmtime(p) <= t for p in _inputs())


def nvcc() -> str:
    exe = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.isfile(exe):
        raise RuntimeError("nvcc not found: the ZTCP CUDA library cannot be built")
    return exe


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile the library unless it is newer than every source; return its path."""
    if not force and up_to_date():
        return LIB_PATH
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc(), *NVCC_FLAGS, "-I", INCLUDE, "-o", tmp, *sources()]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force=True, verbose=True))
