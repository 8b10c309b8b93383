"""Builds libjxrng.so in-tree with nvcc for sm_100a (no GPU needed to build).

    python -m jaxr_b200.build          # or jaxr_b200.build.build()
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "libjxrng.so")
SOURCES = [os.path.join(CSRC, "jxrng.cu")]
# every header the library includes: a change to any of them rebuilds it
HEADERS = sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))) + [
    os.path.join(ROOT, "include", "jxrng.h")]

NVCC_FLAGS = [
    "-O3", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo",
    "-Xcompiler", "-fPIC", "-shared", "-I" + os.path.join(ROOT, "include"),
]


def nvcc():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def up_to_date():
    if not os.path.exists(OUT):
        return False
    t = os.path.getmtime(OUT)
    return all(os.path.getmtime(p) <= t for p in SOURCES + HEADERS + [__file__])


def build(force=False, verbose=False, extra=()):
    if not force and up_to_date():
        return OUT
    cmd = [nvcc(), *NVCC_FLAGS, *extra, "-o", OUT + ".tmp", *SOURCES]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(OUT + ".tmp", OUT)
    return OUT


# ---- XLA typed-FFI handlers (csrc/ffi/jxrng_ffi.cc) -----------------------------------------

FFI_SOURCE = os.path.join(CSRC, "ffi", "jxrng_ffi.cc")
FFI_OUT = os.path.join(HERE, "libjxrng_ffi.so")


FFI_HEADERS = [os.path.join(CSRC, "ffi", "xla_ffi_abi.h"), os.path.join(ROOT, "include", "jxrng.h"),
               os.path.join(ROOT, "include", "jxrng_ffi.h")]


def xla_ffi_include_dir():
    """$XLA_FFI_INCLUDE_DIR when it holds xla/ffi/api/c_api.h (XLA's own FFI header, e.g.
    the copy jaxR vendors for ffi_include_dir()), else None."""
    cand = os.environ.get("XLA_FFI_INCLUDE_DIR")
    if cand and os.path.exists(os.path.join(cand, "xla", "ffi", "api", "c_api.h")):
        return cand
    return None


def build_ffi(force=False, verbose=False):
    """Builds libjxrng_ffi.so (host C++, linked to libjxrng.so) and returns its path.  The
    handlers compile against csrc/ffi/xla_ffi_abi.h, the part of XLA's FFI C API they use;
    with $XLA_FFI_INCLUDE_DIR set they compile against XLA's own c_api.h instead."""
    inc = xla_ffi_include_dir()
    lib = build(verbose=verbose)
    if (not force and os.path.exists(FFI_OUT) and
            all(os.path.getmtime(q) <= os.path.getmtime(FFI_OUT)
                for q in [FFI_SOURCE, lib, __file__] + FFI_HEADERS)):
        return FFI_OUT
    cxx = os.environ.get("CXX_FOR_FFI") or shutil.which("g++") or "g++"
    cmd = [cxx, "-O2", "-std=c++17", "-fPIC", "-shared", "-Wall",
           "-I" + os.path.join(CSRC, "ffi"), "-I" + os.path.join(ROOT, "include")]
    if inc is not None:
        cmd += ["-DJXR_FFI_XLA_HEADER", "-I" + inc]
    cmd += [FFI_SOURCE, "-L" + HERE, "-ljxrng", "-Wl,-rpath,$ORIGIN", "-o", FFI_OUT + ".tmp"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(FFI_OUT + ".tmp", FFI_OUT)
    return FFI_OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
    print(build_ffi(force="--force" in sys.argv, verbose=True))
