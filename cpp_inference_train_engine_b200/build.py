"""Builds the sm_100a backend in place: cpp_inference_train_engine_b200/libmm_cuda.so.

    python -m cpp_inference_train_engine_b200.build

nvcc cross-compiles for sm_100a without a GPU. The CUDA runtime is linked statically and
NCCL is opened at run time, so the library's only CUDA dependency is the driver.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
SRC = os.path.join(HERE, "csrc", "mm_cuda.cu")
OUT = os.path.join(HERE, "libmm_cuda.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def sources():
    d = os.path.join(HERE, "csrc")
    return [os.path.join(d, f) for f in os.listdir(d)] + [
        os.path.join(ROOT, "include", f) for f in os.listdir(os.path.join(ROOT, "include"))]


def up_to_date() -> bool:
    if not os.path.exists(OUT):
        return False
    t = os.path.getmtime(OUT)
    return all(os.path.getmtime(s) <= t for s in sources())


def build(force: bool = False, verbose: bool = True) -> str:
    if not force and up_to_date():
        return OUT
    cmd = [NVCC, *ARCH, "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
           "-Xcompiler", "-fPIC", "-shared", "-cudart", "static", "-Xptxas", "-warn-spills",
           "-I", os.path.join(ROOT, "include"), SRC, "-o", OUT + ".tmp", "-ldl", "-lpthread"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc failed")
    if verbose and r.stderr.strip():
        sys.stderr.write(r.stderr)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    build(force="--force" in sys.argv)
