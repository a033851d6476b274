"""Build gs_xla_ffi.so, the XLA typed-FFI handlers of libgsb200.so, next to
this file. Needs jaxlib's FFI headers (jax.ffi.include_dir()); exits with a
message and status 2 where jax is not installed.

  python jax-gs_b200/xla/build_ffi.py
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
INCLUDE = os.path.join(os.path.dirname(PKG), "include")
LIBDIR = os.path.join(PKG, "gs_b200")
OUT = os.path.join(HERE, "gs_xla_ffi.so")


def ffi_include_dir():
    """jaxlib's FFI header directory, or None without jax."""
    try:
        import jax
    except ImportError:
        return None
    return jax.ffi.include_dir()


def build() -> str:
    inc = ffi_include_dir()
    if inc is None:
        raise RuntimeError("jax is not installed: the XLA FFI handlers cannot be built here")
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cxx = shutil.which("g++") or "g++"
    cmd = [cxx, "-O2", "-std=c++17", "-shared", "-fPIC", "-I" + inc, "-I" + INCLUDE,
           "-I" + os.path.join(cuda, "include"), os.path.join(HERE, "gs_xla_ffi.cc"), "-L" + LIBDIR,
           "-lgsb200", "-Wl,-rpath," + LIBDIR, "-o", OUT]
    subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    try:
        print(build())
    except RuntimeError as e:
        print(e, file=sys.stderr)
        sys.exit(2)
