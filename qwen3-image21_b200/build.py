"""Build recipe of libb200attn.so (sm_100a) — run by ``__graft_entry__.build()``.

The library is built in-tree (``b200attn/libb200attn.so``) with nvcc, static cudart, and
``-gencode arch=compute_100a,code=sm_100a``; ptxas resource usage is written to
``_build/ptxas.log`` next to this file.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "b200attn", "libb200attn.so")
SOURCES = ["attn_fwd.cu", "block_ops.cu", "dequant.cu", "gemm.cu", "host_layout.cpp", "tp.cpp"]
HEADERS = ["ptx.cuh", os.path.join("..", "..", "include", "b200_attn.h"),
           os.path.join("..", "..", "include", "b200_block_ops.h"),
           os.path.join("..", "..", "include", "b200_gguf.h"),
           os.path.join("..", "..", "include", "b200_gemm.h"),
           os.path.join("..", "..", "include", "b200_tp.h")]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, s) for s in SOURCES + HEADERS] + [os.path.abspath(__file__)]
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile the CUDA extension for sm_100a; returns the library path."""
    if not force and not _stale():
        return LIB
    os.makedirs(os.path.join(HERE, "_build"), exist_ok=True)
    cmd = [
        nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo",
        "-std=c++17", "-Xcompiler", "-fPIC,-O3", "-shared", "-cudart", "static",
        "-Xptxas", "-v", "-I", os.path.join(ROOT, "include"),
        "-o", LIB,
    ] + [os.path.join(CSRC, s) for s in SOURCES] + ["-ldl"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    with open(os.path.join(HERE, "_build", "ptxas.log"), "w") as f:
        f.write(" ".join(cmd) + "\n" + res.stdout + res.stderr)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("nvcc failed building libb200attn.so")
    if verbose:
        sys.stdout.write(res.stderr)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
