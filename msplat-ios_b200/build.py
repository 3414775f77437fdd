"""Build libmsplat_b200.so in-tree with nvcc for sm_100a.

    python msplat-ios_b200/build.py            # incremental
    python msplat-ios_b200/build.py --clean    # from scratch

Each .cu file in csrc/ is compiled separately (project.cu with -fmad=false so
its forward math keeps a fixed IEEE rounding sequence; project_bwd.cu, whose
gradients are compared within tolerances, with approximate sqrt/division) and
linked into
lib/libmsplat_b200.so with the CUDA runtime linked statically, so the library
needs only the driver at run time.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIBDIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIBDIR, "libmsplat_b200.so")
REPO = os.path.dirname(HERE)

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
          "-I", os.path.join(REPO, "include"), "-I", CSRC]
PER_FILE = {"project.cu": ["-fmad=false"], "densify.cu": ["-fmad=false"],
            "project_bwd.cu": ["-prec-div=false", "-prec-sqrt=false"]}
HOST_SOURCES = ["model.cpp"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    cu = sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))
    cpp = [f for f in HOST_SOURCES if os.path.exists(os.path.join(CSRC, f))]
    return cu, cpp


def _stale(obj: str, deps) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, clean: bool = False) -> str:
    if clean and os.path.isdir(BUILD):
        shutil.rmtree(BUILD)
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h", ".hpp"))]
    headers += [os.path.join(REPO, "include", f) for f in os.listdir(os.path.join(REPO, "include"))]
    cu, cpp = sources()
    objs = []
    nv = nvcc()
    for f in cu + cpp:
        src = os.path.join(CSRC, f)
        obj = os.path.join(BUILD, f + ".o")
        objs.append(obj)
        if not _stale(obj, [src, __file__] + headers):
            continue
        cmd = [nv] + ARCH + COMMON + PER_FILE.get(f, []) + ["-c", src, "-o", obj]
        if f.endswith(".cpp"):
            cmd = ["g++", "-O3", "-std=c++17", "-fPIC", "-ffp-contract=off", "-fno-fast-math",
                   "-I", os.path.join(REPO, "include"), "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
    if _stale(LIB, objs):
        cmd = [nv] + ARCH + ["-shared", "-cudart", "static", "-o", LIB] + objs + ["-lpthread", "-ldl", "-lrt"]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(verbose=True, clean="--clean" in sys.argv)
    print(LIB)
