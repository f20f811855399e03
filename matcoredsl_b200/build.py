"""Build libmcb.so (the sm_100a kernels + C ABI) in-tree with nvcc.

Usage: ``python -m matcoredsl_b200.build [--force]``. Objects go to
``matcoredsl_b200/_build/``; the shared library to ``matcoredsl_b200/libmcb.so``
so that it travels with the source tree. nvcc cross-compiles for sm_100a; no
GPU is needed to build.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libmcb.so")
NVCC = os.environ.get("MCB_NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden",
    "-I", os.path.join(ROOT, "include"), "-I", CSRC, "--expt-relaxed-constexpr",
    "-ccbin", "/usr/bin/g++",
]
# The strict kernels must never contract a multiply and an add, and must keep
# subnormals (bit-exact with the reference's strict CPU leaf).
STRICT = ["-fmad=false", "-ftz=false", "-prec-div=true", "-prec-sqrt=true"]

SOURCES = {
    "api.cpp": [],
    "strict.cu": STRICT,
    "gemm_tc.cu": [],
    "simt.cu": [],
    "noalloc.cu": [],
    "msm_tc.cu": [],
    "chain_tc.cu": [],
    "fp8.cu": [],
    "region.cu": [],
    "plan.cpp": [],
    "typed.cu": [],
    "comm.cpp": [],
    "peer.cu": [],
}
HEADERS = ["common.cuh", "internal.h", "epilogue.cuh"]


def _newer(src_paths, out):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(p) > t for p in src_paths)


def _compile(name, extra, force):
    src = os.path.join(CSRC, name)
    obj = os.path.join(BUILD, name + ".o")
    deps = [src, os.path.join(ROOT, "include", "mcb.h")] + [os.path.join(CSRC, h) for h in HEADERS]
    if not force and not _newer(deps, obj):
        return obj, None
    cmd = [NVCC] + COMMON + extra + ["-c", src, "-o", obj]
    if name.endswith(".cu"):
        cmd += ["-Xptxas", "-v"] if os.environ.get("MCB_PTXAS_V") else []
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {name}:\n{r.stdout}\n{r.stderr}")
    return obj, (r.stdout + r.stderr).strip() or None


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=min(8, len(SOURCES))) as ex:
        futs = [ex.submit(_compile, n, e, force) for n, e in SOURCES.items()]
        objs = []
        for f in futs:
            obj, log = f.result()
            objs.append(obj)
            if verbose and log:
                print(log)
    if force or _newer(objs, LIB):
        cmd = [NVCC] + ARCH + ["-shared", "-o", LIB] + objs + ["-ccbin", "/usr/bin/g++"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
