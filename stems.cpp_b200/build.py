"""Builds the CUDA library in-tree: stems.cpp_b200/libstems_gpu.so (sm_100a only)."""
from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libstems_gpu.so")
SOURCES = ["kernels.cu", "pair.cu", "split.cu", "plan.cu", "engine.cu", "noalloc.cu", "norm.cu", "convert.cu", "vr.cu", "gguf.cu"]
HEADERS = ["fft.cuh", "frame.cuh", "kernels.h", "plan.h", "engine.h"]
NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
              "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "-shared"]


def nvcc() -> str:
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def _inputs():
    files = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    files.append(os.path.join(HERE, "..", "include", "stems_gpu_v1.h"))
    return files


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(f) <= t for f in _inputs())


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile every .cu of csrc/ into one shared library; returns its path."""
    if not force and up_to_date():
        return LIB
    tmp = LIB + ".tmp"
    cmd = [nvcc(), *NVCC_FLAGS, *[os.path.join(CSRC, f) for f in SOURCES], "-o", tmp]
    res = subprocess.run(cmd, cwd=CSRC, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + res.stdout + res.stderr)
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force=True, verbose=True))
