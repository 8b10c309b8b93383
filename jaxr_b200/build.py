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
HEADERS = sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cuh")) + [
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


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
