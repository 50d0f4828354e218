"""Build libmi_paged.so (sm_100a) in-tree with nvcc.

    python minimal-inference_b200/csrc/build.py [--force]

Compiles every .cu in this directory into one shared library next to the
Python package (``mi_b200/libmi_paged.so``). The CUDA runtime is linked
statically, so the library loads on machines without a GPU (for the
exported-symbol checks) and needs no LD_LIBRARY_PATH on the GPU box.
Rebuilds only when a source or header is newer than the library.
"""
from __future__ import annotations

import argparse
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(os.path.dirname(HERE), "mi_b200")
REPO = os.path.dirname(os.path.dirname(HERE))
LIB = os.path.join(PKG, "libmi_paged.so")
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


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(f) <= t for f in deps())


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB
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
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=True))
