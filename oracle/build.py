"""Builds the CPU oracle (TEST INFRASTRUCTURE, never part of the product path).

    python oracle/build.py            # oracle/liboracle.so (+ oracle/_ref when the reference is present)

1. oracle/liboracle.so   -- the C restatement hyperion_oracle.c (gcc, pthreads).
2. oracle/_ref/libref_fp8.so -- the reference's own `fp8_e4m3_to_fp32`
   (hyperion_fa3_production_final.py:122-141), compiled for the host from the
   reference's source where it lies.  The reference keeps its CUDA code in a
   Python string (`cuda_source`, :49-602); this script reads that string with
   `ast` (the module is never executed), cuts out the one function by brace
   matching and pipes it to gcc on stdin behind a three-line shim that maps
   `__device__` / `__forceinline__` to host C.  Nothing of the reference is
   written into this repository: the only output is the .so under oracle/_ref/.
   The rest of the reference's kernel does not build here (nvcc errors at :206
   and :222) and is not the sign-bit path, so it is not compiled.
"""
from __future__ import annotations

import ast
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_DIR = os.path.join(HERE, "_ref")
REF_SO = os.path.join(REF_DIR, "libref_fp8.so")
REF_MODULE = "hyperion_fa3_production_final.py"


def reference_file() -> str | None:
    """The reference's module inside the checkout named by HYPERION_REFERENCE_DIR, or
    None when the variable is unset or the file is absent (the GPU box has none)."""
    root = os.environ.get("HYPERION_REFERENCE_DIR")
    if not root:
        return None
    path = os.path.join(root, REF_MODULE)
    return path if os.path.exists(path) else None

CFLAGS = ["-O3", "-march=x86-64-v2", "-fPIC", "-shared", "-ffp-contract=off", "-std=gnu11", "-pthread"]


def _cc() -> str:
    return os.environ.get("CC") or shutil.which("gcc") or "cc"


def build_oracle(force: bool = False) -> str:
    src = os.path.join(HERE, "hyperion_oracle.c")
    if not force and os.path.exists(ORACLE_SO) and os.path.getmtime(ORACLE_SO) >= max(
        os.path.getmtime(src), os.path.getmtime(__file__)
    ):
        return ORACLE_SO
    cmd = [_cc(), *CFLAGS, src, "-o", ORACLE_SO + ".tmp", "-lm"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{res.stderr}")
    os.replace(ORACLE_SO + ".tmp", ORACLE_SO)
    return ORACLE_SO


def _reference_cuda_source(path: str) -> str:
    tree = ast.parse(open(path, encoding="utf-8").read(), filename=path)
    for node in tree.body:
        if isinstance(node, ast.Assign) and any(isinstance(t, ast.Name) and t.id == "cuda_source" for t in node.targets):
            if isinstance(node.value, ast.Constant) and isinstance(node.value.value, str):
                return node.value.value
    raise RuntimeError("cuda_source string not found in the reference module")


def _cut_function(src: str, name: str) -> str:
    """Text of the function `name` (from its return type line to its closing brace)."""
    i = src.index(f" {name}(")
    start = src.rfind("\n", 0, src.rfind("\n", 0, i)) + 1  # include the qualifier line above
    j = src.index("{", i)
    depth = 0
    for k in range(j, len(src)):
        if src[k] == "{":
            depth += 1
        elif src[k] == "}":
            depth -= 1
            if depth == 0:
                return src[start : k + 1]
    raise RuntimeError(f"unbalanced braces in {name}")


SHIM = "#include <stdint.h>\n#include <math.h>\n#define __device__\n#define __forceinline__ static inline\n"
EXPORT = "\nfloat ref_fp8_e4m3_to_fp32(uint8_t x) { return fp8_e4m3_to_fp32(x); }\n"


def build_ref(force: bool = False) -> str | None:
    """Compiles the reference's FP8 decode; None when the reference is absent."""
    ref_file = reference_file()
    if ref_file is None:
        return REF_SO if os.path.exists(REF_SO) else None
    if not force and os.path.exists(REF_SO) and os.path.getmtime(REF_SO) >= os.path.getmtime(__file__):
        return REF_SO
    os.makedirs(REF_DIR, exist_ok=True)
    func = _cut_function(_reference_cuda_source(ref_file), "fp8_e4m3_to_fp32")
    cmd = [_cc(), "-O2", "-fPIC", "-shared", "-x", "c", "-", "-o", REF_SO + ".tmp", "-lm"]
    res = subprocess.run(cmd, input=SHIM + func + EXPORT, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"reference fp8 build failed:\n{res.stderr}")
    os.replace(REF_SO + ".tmp", REF_SO)
    return REF_SO


if __name__ == "__main__":
    force = "--force" in sys.argv
    print(build_oracle(force))
    print(build_ref(force))
