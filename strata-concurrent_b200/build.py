"""Build libstrata_kv.so (the CUDA kernels + C ABI) in-tree for sm_100a.

    python strata-concurrent_b200/build.py          # incremental
    python strata-concurrent_b200/build.py --force  # rebuild

nvcc cross-compiles without a GPU, so this runs on the build host and the .so travels with the tree.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(HERE, "libstrata_kv.so")

CUDA_SOURCES = ["skv_copy.cu", "skv_abi.cu", "kv_stream.cu"]
# the C++ drop-in layer (strata::core API), host code on top of the C ABI
HOST_SOURCES = ["host/pinned.cpp", "host/transfer.cpp", "host/conversation_snapshot.cpp", "host/conversation_state.cpp",
                "host/conversation_wire.cpp", "host/conversation_wire_device.cpp", "host/handoff.cpp",
                "host/handoff_device.cpp", "host/handoff_schedule.cpp"]
CXX = os.environ.get("CXX", "g++")
CXXFLAGS = ["-std=c++20", "-O2", "-fPIC", "-Wall", "-Wextra", "-Wno-unused-parameter", "-I", INCLUDE, "-I", CSRC,
            "-I", "/usr/local/cuda/include"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2,-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-I", INCLUDE, "-I", CSRC]


def _newer(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str]) -> None:
    print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def build(force: bool = False, verbose_ptxas: bool = False) -> str:
    deps = [os.path.join(d, f) for d in (CSRC, os.path.join(CSRC, "host"), os.path.join(INCLUDE, "strata_kv"))
            for f in os.listdir(d)] + [os.path.join(INCLUDE, "strata_kv.h")]
    if not force and not _newer(LIB, deps):
        return LIB
    objs = []
    for src in CUDA_SOURCES:
        obj = os.path.join(CSRC, src.replace(".cu", ".o"))
        cmd = [NVCC, *ARCH, *FLAGS, "-c", os.path.join(CSRC, src), "-o", obj]
        if verbose_ptxas:
            cmd.insert(1, "-Xptxas=-v")
        _run(cmd)
        objs.append(obj)
    for src in HOST_SOURCES:
        obj = os.path.join(CSRC, src.replace("/", "_").replace(".cpp", ".o"))
        _run([CXX, *CXXFLAGS, "-c", os.path.join(CSRC, src), "-o", obj])
        objs.append(obj)
    _run([NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-lcudart"])
    for o in objs:
        os.remove(o)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose_ptxas=a.ptxas_v))
    sys.exit(0)
