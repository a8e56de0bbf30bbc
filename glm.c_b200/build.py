"""Build the in-tree CUDA library libglm_cuda.so for sm_100a with nvcc.

The library is the product: the C-ABI of include/glm_cuda.h over the
hand-written kernels in csrc/. It is built in place (next to this file) so it
travels with the source tree; nothing is installed into site-packages.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(PKG, "libglm_cuda.so")

SOURCES = ["glm_cuda.cu", "moe_decode.cu", "moe_persistent.cu", "q80_matvec.cu", "moe_noalloc.cu", "decoder.cu", "moe_prefill.cu", "checkpoint.cu"]
HEADERS = ["glm_internal.h", "q80_common.cuh", "route_common.cuh", "glm_cuda.map"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-O2",
    "--expt-relaxed-constexpr",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _inputs():
    return [os.path.join(CSRC, s) for s in SOURCES + HEADERS] + [os.path.join(INCLUDE, "glm_cuda.h"), __file__]


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(p) <= t for p in _inputs())


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> str:
    if not force and not ptxas_info and up_to_date():
        return LIB
    host_cc = "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else None
    cmd = [nvcc(), *NVCC_FLAGS, "-I", INCLUDE, "-I", CSRC, "-shared", "-o", LIB + ".tmp",
           "-Xlinker", "--version-script=" + os.path.join(CSRC, "glm_cuda.map")]
    if host_cc:
        cmd += ["-ccbin", host_cc]
    if ptxas_info:
        cmd += ["-Xptxas", "-v"]
    cmd += [os.path.join(CSRC, s) for s in SOURCES]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
    if ptxas_info or verbose:
        sys.stderr.write(r.stdout + r.stderr)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_info="--ptxas" in sys.argv)
    print(LIB)
