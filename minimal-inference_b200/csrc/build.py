"""Build libmi_paged.so (sm_100a) in-tree with nvcc.

    python minimal-inference_b200/csrc/build.py [--force]

Compiles every .cu in this directory into one shared library next to the
Python package (``mi_b200/libmi_paged.so``). The CUDA runtime is linked
statically, so the library loads on machines without a GPU (for the
exported-symbol checks) and needs no LD_LIBRARY_PATH on the GPU box.
Rebuilds only when the sources, headers or flags differ from those the
library was built from (a SHA-256 of their contents, kept next to the
library), so a checkout that leaves old mtimes cannot keep a stale build.
"""
from __future__ import annotations

import argparse
import glob
import hashlib
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(os.path.dirname(HERE), "mi_b200")
REPO = os.path.dirname(os.path.dirname(HERE))
LIB = os.path.join(PKG, "libmi_paged.so")
STAMP = LIB + ".sha256"
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
    "-cudart", "static", "--expt-relaxed-constexpr",
]


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(HERE, "*.cu")))


def deps() -> list[str]:
    return (sources() + glob.glob(os.path.join(HERE, "*.cuh"))
            + glob.glob(os.path.join(REPO, "include", "*.h")))


def source_hash() -> str:
    """SHA-256 over the flags and the names and contents of every source and header."""
    h = hashlib.sha256(" ".join(NVCC_FLAGS).encode())
    for f in sorted(deps()):
        h.update(os.path.basename(f).encode())
        with open(f, "rb") as fh:
            h.update(fh.read())
    return h.hexdigest()


def up_to_date() -> bool:
    if not (os.path.exists(LIB) and os.path.exists(STAMP)):
        return False
    with open(STAMP) as f:
        return f.read().strip() == source_hash()


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    digest = source_hash()
    nvcc = os.environ.get("NVCC", "nvcc")
    tmp = LIB + ".tmp"
    cmd = [nvcc, *NVCC_FLAGS, "-I", os.path.join(REPO, "include"), "-o", tmp, *sources()]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc failed building libmi_paged.so")
    os.replace(tmp, LIB)
    with open(STAMP, "w") as f:
        f.write(digest + "\n")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=True))
