"""Build libeg2_b200.so in-tree for sm_100a (nvcc cross-compiles without a GPU).

    python embeddinggemma2-amdkfd_b200/build.py [--force]
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libeg2_b200.so")
SOURCES = ["kernels.cu", "executor.cu", "gguf.cpp"]
HEADERS = ["common.cuh", "q8gemm.cuh", "q8vnni.cuh", "exact.cuh", "ple.cuh", "rowops.cuh", "attention.cuh", "attention_tc.cuh",
           "opsabi.cuh", "launch.h", "ref_expf.h", "ref_tanhf.h"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-lineinfo",
         "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall"]


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    inc = os.path.join(os.path.dirname(HERE), "include")
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS] + [
        os.path.join(inc, f) for f in os.listdir(inc)]
    return any(os.path.getmtime(p) > t for p in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not _stale():
        return LIB
    objs = []
    for src in SOURCES:
        obj = os.path.join(CSRC, "_build", src + ".o")
        os.makedirs(os.path.dirname(obj), exist_ok=True)
        cmd = [NVCC, *FLAGS, "-c", os.path.join(CSRC, src), "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objs.append(obj)
    tmp = LIB + ".tmp"
    subprocess.run([NVCC, *FLAGS, "-shared", *objs, "-o", tmp], check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
