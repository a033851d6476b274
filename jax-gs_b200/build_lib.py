"""Build libgsb200.so (all CUDA kernels + the C ABI) in-tree for sm_100a.

Usage: python jax-gs_b200/build_lib.py [--force] [--verbose]

The library is compiled with nvcc directly (no torch extension machinery):
each .cu file becomes an object, then one shared library is linked against
the shared CUDA runtime, so that it shares the runtime state (current device,
streams) of whatever framework loaded it first (torch, XLA).
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
OUT_DIR = os.path.join(HERE, "gs_b200")
LIB_PATH = os.path.join(OUT_DIR, "libgsb200.so")
BUILD_DIR = os.path.join(HERE, "_build")

SOURCES = [
    "gs_preprocess.cu",
    "gs_sort.cu",
    "gs_raster.cu",
    "gs_train.cu",
    "gs_ssim.cu",
    "gs_loss.cu",
    "gs_density.cu",
    "gs_2dgs.cu",
    "gs_capi.cu",
    "gs_timing.cu",
    "gs_noalloc.cu",
    "gs_dp.cu",
]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-I" + INCLUDE,
]


def _nvcc() -> str:
    cand = [os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"]
    for c in cand:
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def _cuda_lib_dir(nvcc: str) -> str:
    root = os.path.dirname(os.path.dirname(os.path.realpath(nvcc)))
    for d in ("lib64", "targets/x86_64-linux/lib"):
        p = os.path.join(root, d)
        if os.path.isdir(p):
            return p
    return "/usr/local/cuda/lib64"


def _newest_input_mtime() -> float:
    paths = [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
    paths += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE)]
    paths.append(os.path.abspath(__file__))
    return max(os.path.getmtime(p) for p in paths)


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> str:
    """Compile the library if any source is newer than it; return its path."""
    if (not force and os.path.exists(LIB_PATH)
            and os.path.getmtime(LIB_PATH) >= _newest_input_mtime()):
        return LIB_PATH
    nvcc = _nvcc()
    os.makedirs(BUILD_DIR, exist_ok=True)
    objs = []
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []
    for src in SOURCES:
        obj = os.path.join(BUILD_DIR, src.replace(".cu", ".o"))
        cmd = [nvcc, *ARCH_FLAGS, *COMMON_FLAGS, *extra, "-c", os.path.join(CSRC, src), "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{res.stdout}\n{res.stderr}")
        if verbose or ptxas_verbose:
            sys.stdout.write(res.stdout + res.stderr)
        objs.append(obj)
    libdir = _cuda_lib_dir(nvcc)
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-cudart", "shared", "-o", tmp, *objs,
           "-Xlinker", "-rpath," + libdir]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas", action="store_true", help="print -Xptxas -v register/smem usage")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose, ptxas_verbose=a.ptxas))
