"""Builds the CUDA library in-tree for sm_100a.

    python -m polarquant_b200.build [--force]

Compiles polarquant_b200/csrc/all.cu (one translation unit that includes every
kernel file) with nvcc into polarquant_b200/_lib/libpolarquant_b200.so.  The
build is skipped when the library is newer than every source file.
"""

from __future__ import annotations

import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
SRC = os.path.join(HERE, "csrc", "all.cu")
OUT = os.path.join(HERE, "_lib", "libpolarquant_b200.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
]


def sources():
    return (glob.glob(os.path.join(HERE, "csrc", "*.cu")) +
            glob.glob(os.path.join(HERE, "csrc", "*.cuh")) +
            glob.glob(os.path.join(ROOT, "include", "*.h")))


def up_to_date() -> bool:
    if not os.path.exists(OUT):
        return False
    t = os.path.getmtime(OUT)
    return all(os.path.getmtime(s) <= t for s in sources())


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if c and (os.path.isabs(c) and os.path.exists(c) or not os.path.isabs(c)):
            return c
    return "nvcc"


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return OUT
    os.makedirs(os.path.dirname(OUT), exist_ok=True)
    tmp = OUT + f".tmp{os.getpid()}"
    cmd = [nvcc()] + NVCC_FLAGS + ["-o", tmp, SRC]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
