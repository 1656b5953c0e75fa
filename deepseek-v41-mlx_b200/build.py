"""Build libdsv41q.so (the C-ABI CUDA library) in-tree for sm_100a.

    python deepseek-v41-mlx_b200/build.py [--verbose-ptxas]

nvcc cross-compiles without a GPU.  The library links the CUDA runtime
statically and resolves cuTensorMapEncodeTiled through cudaGetDriverEntryPoint,
so it loads on a machine without a GPU (compute calls then fail loudly).
"""

from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
SRC = os.path.join(HERE, "csrc", "dsv41q.cu")
OUT = os.path.join(HERE, "libdsv41q.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")


def sources():
    d = os.path.join(HERE, "csrc")
    return [os.path.join(d, f) for f in sorted(os.listdir(d)) if f.endswith((".cu", ".cuh"))] + \
        [os.path.join(ROOT, "include", "dsv41q.h")]


def up_to_date() -> bool:
    if not os.path.exists(OUT):
        return False
    t = os.path.getmtime(OUT)
    return all(os.path.getmtime(s) <= t for s in sources())


def build(verbose_ptxas: bool = False, force: bool = False) -> str:
    if not force and up_to_date():
        return OUT
    cmd = [NVCC, "-O3", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo",
           "-Xcompiler", "-fPIC", "-shared", "--expt-relaxed-constexpr",
           "-I", os.path.join(ROOT, "include"), "-I", os.path.join(HERE, "csrc"),
           "-o", OUT + ".tmp", SRC]
    if verbose_ptxas:
        cmd[1:1] = ["-Xptxas", "-v"]
    subprocess.run(cmd, check=True)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(verbose_ptxas="--verbose-ptxas" in sys.argv, force=True))
