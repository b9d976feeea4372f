"""Build libmfftb200.so in-tree (mfft_bench_b200/lib/) for sm_100a.

    python mfft_bench_b200/build.py          # incremental
    python mfft_bench_b200/build.py --clean

nvcc cross-compiles without a GPU, so this runs on the CPU-only build host;
the resulting .so travels with the repository snapshot to the GPU box.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OBJ = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "lib")
SO = os.path.join(LIB, "libmfftb200.so")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CU_FLAGS = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
                   "-Xcompiler", "-Wall"]
CXX_FLAGS = ["-O2", "-std=c++17", "-fPIC", "-Wall", "-Wextra"]
C_FLAGS = ["-O2", "-std=gnu11", "-fPIC", "-Wall", "-Wextra", "-fopenmp"]

CU_SOURCES = ["pointwise.cu", "pack.cu", "fwd.cu", "inv.cu", "engine.cu", "noalloc.cu"]
CXX_SOURCES = ["plan.cpp"]
C_SOURCES = ["refapi.c"]


def _headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    inc = os.path.join(ROOT, "include")
    hs += [os.path.join(inc, f) for f in os.listdir(inc) if f.endswith(".h")]
    return hs


def _stale(obj, src, headers):
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return os.path.getmtime(src) > t or any(os.path.getmtime(h) > t for h in headers)


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"build failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return r.stderr


def build(verbose: bool = False) -> str:
    if not os.path.exists(NVCC):
        raise RuntimeError(f"nvcc not found at {NVCC}")
    os.makedirs(OBJ, exist_ok=True)
    os.makedirs(LIB, exist_ok=True)
    headers = _headers()
    jobs, objs = [], []
    for f in CU_SOURCES:
        src, obj = os.path.join(CSRC, f), os.path.join(OBJ, f + ".o")
        objs.append(obj)
        if _stale(obj, src, headers):
            jobs.append([NVCC] + CU_FLAGS + ["-c", src, "-o", obj])
    for f in CXX_SOURCES:
        src, obj = os.path.join(CSRC, f), os.path.join(OBJ, f + ".o")
        objs.append(obj)
        if _stale(obj, src, headers):
            jobs.append(["g++"] + CXX_FLAGS + ["-c", src, "-o", obj])
    for f in C_SOURCES:
        src, obj = os.path.join(CSRC, f), os.path.join(OBJ, f + ".o")
        objs.append(obj)
        if _stale(obj, src, headers):
            jobs.append(["gcc"] + C_FLAGS + ["-c", src, "-o", obj])
    with cf.ThreadPoolExecutor(max_workers=max(1, os.cpu_count() or 1)) as ex:
        for err in ex.map(_run, jobs):
            if verbose and err:
                print(err, file=sys.stderr)
    newest = max(os.path.getmtime(o) for o in objs)
    if not os.path.exists(SO) or os.path.getmtime(SO) < newest:
        _run([NVCC] + ARCH + ["-shared", "-o", SO] + objs +
             ["-lgomp", "-Xlinker", "--no-undefined", "-Xlinker", "-rpath=$ORIGIN"])
    return SO


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--clean", action="store_true")
    ap.add_argument("-v", action="store_true")
    a = ap.parse_args()
    if a.clean:
        shutil.rmtree(OBJ, ignore_errors=True)
        shutil.rmtree(LIB, ignore_errors=True)
    print(build(verbose=a.v))


if __name__ == "__main__":
    main()
