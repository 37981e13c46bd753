"""Build libnanokv.so in-tree with nvcc for sm_100a (no torch build machinery).

    python -m <package>.build        or   build_library() from Python

The shared library exports exactly the C ABI of include/nanokv.h.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libnanokv.so")
SOURCES = ["nkv_capi.cu", "nkv_select.cu", "nkv_attend.cu", "nkv_store.cu", "nkv_prefill.cu", "nkv_prefill_tc.cu",
           "nkv_model.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc():
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.isabs(cand) and os.path.exists(cand) or not os.path.isabs(cand)):
            return cand
    raise RuntimeError("nvcc not found")


def build_library(verbose: bool = False, extra=(), checked: bool = False) -> str:
    """checked=True builds libnanokv_checked.so with -DNKV_CHECKED (bounds checks
    that record a bad access in the workspace error word instead of making it)."""
    srcs = [os.path.join(CSRC, s) for s in SOURCES if os.path.exists(os.path.join(CSRC, s))]
    objdir = os.path.join(ROOT, "_build", "checked" if checked else "release")
    if checked:
        extra = (*extra, "-DNKV_CHECKED")
    os.makedirs(objdir, exist_ok=True)
    objs = []
    for src in srcs:
        obj = os.path.join(objdir, os.path.basename(src) + ".o")
        deps = [src] + [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
        deps.append(os.path.join(ROOT, "include", "nanokv.h"))
        if not os.path.exists(obj) or os.path.getmtime(obj) < max(os.path.getmtime(d) for d in deps):
            cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                   "-I", os.path.join(ROOT, "include"), "-c", src, "-o", obj, *extra]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
                print(" ".join(cmd))
            subprocess.run(cmd, check=True)
        objs.append(obj)
    lib = LIB.replace(".so", "_checked.so") if checked else LIB
    cmd = [nvcc(), *ARCH, "-shared", "-o", lib, *objs, "-lcudart"]
    subprocess.run(cmd, check=True)
    return lib


if __name__ == "__main__":
    print(build_library(verbose="-v" in sys.argv, checked="--checked" in sys.argv))
