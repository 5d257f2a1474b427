"""Build librapier_b200.so in-tree with nvcc for sm_100a (no torch extension, no JIT cache).

    python -m rapier_b200.build          # incremental: rebuilds objects whose sources changed

The library is plain C-ABI (include/rapier_b200.h); the CUDA runtime is linked statically, so it loads
on a machine without a GPU (entry points then return RK_ECUDA).
"""
from __future__ import annotations

import hashlib
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OBJ = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "librapier_b200.so")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# --fmad=false: device code never fuses a multiply and an add unless it says so (__fmaf_rn), the same rule as
# the CPU oracle's -ffp-contract=off, so both compute every fp32 expression with the same roundings.
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--fmad=false", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
         "-Xcompiler", "-ffp-contract=off",
         "--expt-relaxed-constexpr", "-I" + os.path.join(ROOT, "include")]


def _sources():
    return sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))


def _headers_digest() -> str:
    h = hashlib.sha256()
    for d in (CSRC, os.path.join(ROOT, "include")):
        for f in sorted(os.listdir(d)):
            if f.endswith((".cuh", ".h")):
                with open(os.path.join(d, f), "rb") as fh:
                    h.update(f.encode() + fh.read())
    return h.hexdigest()[:16]


def _compile(src: str, hdr: str, verbose: bool) -> str:
    path = os.path.join(CSRC, src)
    with open(path, "rb") as fh:
        digest = hashlib.sha256(fh.read() + hdr.encode() + " ".join(ARCH + FLAGS).encode()).hexdigest()[:16]
    obj = os.path.join(OBJ, f"{src[:-3]}.{digest}.o")
    if not os.path.exists(obj):
        for old in os.listdir(OBJ):
            if old.startswith(src[:-3] + ".") and old.endswith(".o"):
                os.remove(os.path.join(OBJ, old))
        cmd = [NVCC, *ARCH, *FLAGS, "-c", path, "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return obj


def build(verbose: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    hdr = _headers_digest()
    srcs = _sources()
    with ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, hdr, verbose), srcs))
    newest = max(os.path.getmtime(o) for o in objs)
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < newest:
        cmd = [NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-cudart", "static", "-lpthread", "-ldl", "-lrt"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    build_serve(verbose)
    return LIB


SERVE_SRC = os.path.join(PKG, "serve", "rapier_serve.cpp")
SERVE_BIN = os.path.join(PKG, "rapier_serve")


def build_serve(verbose: bool = False) -> str:
    """The --serve host binary (C++, the C-ABI only), linked to the in-tree library by rpath."""
    deps = [SERVE_SRC, LIB, os.path.join(ROOT, "include", "rapier_b200.h")]
    if os.path.exists(SERVE_BIN) and os.path.getmtime(SERVE_BIN) >= max(os.path.getmtime(d) for d in deps):
        return SERVE_BIN
    cxx = os.environ.get("CXX", "g++")
    cmd = [cxx, "-O2", "-std=c++17", "-Wall", "-I" + os.path.join(ROOT, "include"), SERVE_SRC, "-o", SERVE_BIN,
           "-L" + PKG, "-l:librapier_b200.so", "-Wl,-rpath,$ORIGIN"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    return SERVE_BIN


if __name__ == "__main__":
    build(verbose="-q" not in sys.argv)
    print(LIB)
