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
           os.path.join(HERE, "csrc", "schedule.cpp"), os.path.join(HERE, "csrc", "storage.cpp")]
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


ENGINE_LIB = os.path.join(HERE, "libb2d_engine.so")
ENGINE_TEST = os.path.join(HERE, "test_engine")
HOST = os.path.join(HERE, "host")


def build_host(force: bool = False, verbose: bool = False) -> None:
    """The audio.cpp-facing C++ classes (host/engine_b200.*) as libb2d_engine.so, and their C++ test."""
    srcs = [os.path.join(HOST, f) for f in ("engine_b200.cpp", "engine_b200.h")]
    newest = max(os.path.getmtime(p) for p in srcs + [LIB, os.path.join(HOST, "test_engine.cpp")])
    if not force and os.path.exists(ENGINE_TEST) and os.path.exists(ENGINE_LIB) and \
            min(os.path.getmtime(ENGINE_LIB), os.path.getmtime(ENGINE_TEST)) >= newest:
        return
    common = ["g++", "-std=c++17", "-O2", "-fPIC", "-Wall"]
    cmds = [common + ["-shared", "-o", ENGINE_LIB, os.path.join(HOST, "engine_b200.cpp"), "-L" + HERE, "-lb200diff",
                      "-Wl,-rpath,$ORIGIN"],
            common + ["-o", ENGINE_TEST, os.path.join(HOST, "test_engine.cpp"), "-L" + HERE, "-lb2d_engine",
                      "-lb200diff", "-Wl,-rpath,$ORIGIN"]]
    for cmd in cmds:
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)


def build(force: bool = False, verbose: bool = False) -> str:
    if force or not up_to_date():
        cmd = [nvcc()] + NVCC_FLAGS + ["-o", LIB + ".tmp"] + SOURCES
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
        os.replace(LIB + ".tmp", LIB)
    build_host(force, verbose)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
