"""Builds libhyperion_b200.so in-tree with nvcc for sm_100a only.

    python hyperion-fa3-kernel-_b200/build.py [--force]

The library is a plain C-ABI shared object (include/hyperion_b200.h): no torch
types, CUDA runtime linked statically, so it loads into any process that has a
CUDA driver.  Output: hyperion-fa3-kernel-_b200/hyperion_b200/libhyperion_b200.so.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "hyperion_b200", "libhyperion_b200.so")
INCLUDE = os.path.join(REPO, "include")

SOURCES = ["capi.cu"]
HEADERS = ["common.cuh", "row_kernel.cuh", "row_group_kernel.cuh", "row_mma_kernel.cuh", "tile_kernel.cuh", "tcgen05.cuh", "kv_write.cuh",
           "launch_table.h"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "--expt-relaxed-constexpr",
    "-cudart", "static",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale() -> bool:
    if not os.path.exists(OUT):
        return True
    out_t = os.path.getmtime(OUT)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS] + [os.path.join(INCLUDE, "hyperion_b200.h"), __file__]
    return any(os.path.getmtime(d) > out_t for d in deps if os.path.exists(d))


def build(force: bool = False, verbose: bool = False, ptxas_v: bool = False) -> str:
    if not force and not _stale():
        return OUT
    cmd = [nvcc(), *NVCC_FLAGS, "-I", INCLUDE, "-I", CSRC]
    if ptxas_v:
        cmd += ["-Xptxas", "-v"]
    cmd += [os.path.join(CSRC, s) for s in SOURCES] + ["-o", OUT + ".tmp"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if ptxas_v or verbose:
        sys.stderr.write(res.stderr)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print registers / spills / smem per kernel")
    a = ap.parse_args()
    print(build(force=a.force, verbose=True, ptxas_v=a.ptxas_v))
