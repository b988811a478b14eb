"""Build ``lib/libswa_attn.so`` (the C-ABI library) from ``csrc/*.cu`` for sm_100a.

    python flashattention-gpt-oss-finetuning_b200/build.py [--force] [--verbose]

nvcc compiles each translation unit in parallel to an object under ``_build/`` and links
them into one shared library that depends only on the CUDA runtime (no torch).  A unit is
rebuilt when it or any header in ``csrc/`` or ``include/`` is newer than its object.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(PKG_DIR, "_build")
LIB_DIR = os.path.join(PKG_DIR, "lib")
LIB = os.path.join(LIB_DIR, "libswa_attn.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-I", INCLUDE, "-I", CSRC,
]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libswa_attn.so")
    return cand


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))


def _stale(obj: str, src: str, headers) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(f) > t for f in [src, *headers])


def _compile(src: str, obj: str, verbose: bool, extra=()):
    cmd = [_nvcc(), *NVCC_FLAGS, *extra, "-c", src, "-o", obj]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
    return r.stderr


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    headers = _headers()
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    jobs = []
    for s in srcs:
        obj = os.path.join(BUILD, os.path.basename(s)[:-3] + ".o")
        if force or ptxas_verbose or _stale(obj, s, headers):
            jobs.append((s, obj))
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            futs = {ex.submit(_compile, s, o, verbose, extra): s for s, o in jobs}
            for f in cf.as_completed(futs):
                msg = f.result()
                if ptxas_verbose and msg:
                    print(f"== {os.path.basename(futs[f])}\n{msg}")
    objs = [os.path.join(BUILD, os.path.basename(s)[:-3] + ".o") for s in srcs]
    if force or jobs or not os.path.exists(LIB) or any(
            os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        cmd = [_nvcc(), *ARCH, "-shared", "-o", LIB, *objs, "-lcudart"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.verbose, a.ptxas_verbose))
    sys.exit(0)
