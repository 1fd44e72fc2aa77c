"""Builds the CUDA library in-tree: ``wavo_b200/libwavo_cuda.so`` (for ctypes and C/C++ callers)
and ``wavo_b200/libwavo_cuda.a`` (for a static link from the reference's Rust crate), both for
sm_100a only.

    python -m wavo_b200.build          # or: from wavo_b200.build import build; build()
"""

from __future__ import annotations

import hashlib
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
SOURCES = ["wavo_cuda.cu", "gemm.cu", "attention.cu", "attention_fa.cu", "decode.cu", "selftest.cu",
           "encoder.cu", "decoder.cu", "gguf.cu", "frontend.cu"]
HEADERS = ["ptx.cuh", "kernels.cuh", "softmax.cuh", "gguf.cuh"]
SO = os.path.join(HERE, "libwavo_cuda.so")
STATIC = os.path.join(HERE, "libwavo_cuda.a")
STAMP = os.path.join(HERE, ".libwavo_cuda.stamp")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xptxas", "-v"]


def _digest() -> str:
    h = hashlib.sha256()
    for f in SOURCES + HEADERS:
        with open(os.path.join(CSRC, f), "rb") as fh:
            h.update(fh.read())
    with open(os.path.join(INCLUDE, "wavo_cuda.h"), "rb") as fh:
        h.update(fh.read())
    h.update(" ".join(ARCH + FLAGS).encode())
    return h.hexdigest()


def up_to_date() -> bool:
    if not (os.path.exists(SO) and os.path.exists(STATIC) and os.path.exists(STAMP)):
        return False
    with open(STAMP) as fh:
        return fh.read().strip() == _digest()


def build(force: bool = False, verbose: bool = False) -> str:
    """Compiles the library unless it is up to date; returns the .so path."""
    if not force and up_to_date():
        return SO
    objdir = os.path.join(os.path.dirname(HERE), "_build", "obj")
    os.makedirs(objdir, exist_ok=True)
    objs = []
    for src in SOURCES:
        obj = os.path.join(objdir, src.replace(".cu", ".o"))
        cmd = [NVCC, *ARCH, *FLAGS, "-I", INCLUDE, "-c", os.path.join(CSRC, src), "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if verbose or r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}")
        objs.append(obj)
    tmp = SO + ".tmp"
    r = subprocess.run([NVCC, *ARCH, "-shared", "-o", tmp, *objs], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("link failed: " + r.stdout + r.stderr)
    os.replace(tmp, SO)
    if os.path.exists(STATIC):
        os.remove(STATIC)
    r = subprocess.run([NVCC, *ARCH, "-lib", "-o", STATIC, *objs], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("archive failed: " + r.stdout + r.stderr)
    with open(STAMP, "w") as fh:
        fh.write(_digest())
    return SO


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
