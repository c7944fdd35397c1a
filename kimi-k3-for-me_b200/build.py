"""Build libk3gpu.so (the CUDA C-ABI library) in-tree for sm_100a with nvcc.

The library is plain CUDA C++ behind ``include/k3gpu.h`` (extern "C", device pointers and
sizes only); nothing here depends on torch. ``python kimi-k3-for-me_b200/build.py``
rebuilds whatever is out of date; ``--force`` rebuilds everything.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OBJ = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libk3gpu.so")
SHIM = os.path.join(PKG, "libk3shim.so")   # the reference's host-pointer k3_* names over LIB
SHIM_OPS = os.path.join(PKG, "libk3shim_ops.so")   # the same without k3_router (the op suite's gate)
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-I" + os.path.join(ROOT, "include"), "-I" + CSRC]
SOURCES = ["abi.cu", "router.cu", "moe.cu", "moe_mma.cu", "moe_tc.cu", "kda.cu", "mla.cu", "accept.cu",
           "norm.cu", "mmw.cu", "layer.cu", "ep.cu", "draft.cu", "st.cu", "state.cu",
           "loop.cu", "kda_chunk.cu", "model.cu"]


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    headers.append(os.path.join(ROOT, "include", "k3gpu.h"))
    objs = []
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(OBJ, src.replace(".cu", ".o"))
        objs.append(o)
        if force or _stale(o, [s] + headers):
            cmd = [NVCC, *ARCH, *FLAGS, "-dc", s, "-o", o]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
            subprocess.run(cmd, check=True)
    if force or _stale(LIB, objs):
        subprocess.run([NVCC, *ARCH, "-shared", "-Xcompiler", "-fPIC", *objs, "-o", LIB,
                        "-lcudart"], check=True)
    shim_src = os.path.join(CSRC, "shim.cu")
    for out, extra in ((SHIM, []), (SHIM_OPS, ["-DK3SHIM_NO_ROUTER"])):
        if force or _stale(out, [shim_src, LIB] + headers):
            subprocess.run([NVCC, *ARCH, *FLAGS, *extra, "-shared", shim_src, "-o", out, "-L" + PKG, "-lk3gpu",
                            "-Xlinker", "-rpath,$ORIGIN", "-lcudart"], check=True)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true", help="print ptxas register usage")
    a = ap.parse_args()
    print(build(a.force, a.verbose))
    sys.exit(0)
