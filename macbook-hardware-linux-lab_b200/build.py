"""Builds the sm_100a CUDA library in-tree: csrc/*.cu + csrc/*.cpp -> libgqa_b200.so.

nvcc cross-compiles for sm_100a without a GPU.  The library links the CUDA
runtime statically and exports only the C ABI of include/gqa.h.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libgqa_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-fvisibility=hidden",
    "-Xptxas", "-warn-spills",
]


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(HERE, "csrc", "*.cu")) +
                  glob.glob(os.path.join(HERE, "csrc", "*.cpp")))


# The same sources with the split kernel's phase trace compiled in (profiling).
TRACE_LIB = os.path.join(HERE, "libgqa_b200_trace.so")


def needs_rebuild(lib: str = LIB) -> bool:
    if not os.path.exists(lib):
        return True
    t = os.path.getmtime(lib)
    deps = sources() + glob.glob(os.path.join(HERE, "csrc", "*.cuh")) + [
        os.path.join(REPO, "include", "gqa.h")]
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False, phase_trace: bool = False) -> str:
    lib = TRACE_LIB if phase_trace else LIB
    if not force and not needs_rebuild(lib):
        return lib
    tmp = lib + ".tmp"
    extra = ["-DGQA_PHASE_TRACE"] if phase_trace else []
    cmd = [NVCC, *NVCC_FLAGS, *extra, "-I", os.path.join(REPO, "include"), "-shared", "-o", tmp,
           *sources()]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, lib)
    return lib


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True,
                phase_trace="--phase-trace" in sys.argv))
