"""Builds libb200diff.so (the C-ABI CUDA library) in-tree for sm_100a with nvcc.

    python audio.cpp_b200/build.py

Sources: csrc/api.cu (C ABI + runtimes), csrc/schedule.cpp (host scheduler),
headers csrc/*.cuh and include/b200diff.h.  No torch, no JIT cache: the .so
lands next to this file so it travels with the repository snapshot.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "libb200diff.so")
SOURCES = [os.path.join(HERE, "csrc", "api.cu"), os.path.join(HERE, "csrc", "noalloc.cu"),
           os.path.join(HERE, "csrc", "schedule.cpp")]
DEPS = SOURCES + [os.path.join(HERE, "csrc", f) for f in os.listdir(os.path.join(HERE, "csrc"))] + [
    os.path.join(os.path.dirname(HERE), "include", "b200diff.h")]

NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
              "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "-shared"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.exists(cand) or cand == "nvcc"):
            return cand
    return "nvcc"


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(p) <= t for p in DEPS if os.path.exists(p))


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    cmd = [nvcc()] + NVCC_FLAGS + ["-o", LIB + ".tmp"] + SOURCES
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
