"""Build the detkernels_b200 shared library (sm_100a) in-tree.

    python -m detkernels_b200.build          # -> detkernels_b200/libdetkernels_b200.so

The library is a single CUDA translation unit (csrc/dk_lib.cu) compiled with
nvcc for `sm_100a` only.  It links the CUDA runtime statically and reaches the
driver API (tensor-map encoding) through cudaGetDriverEntryPointByVersion, so
the .so loads on a machine without a GPU driver (symbol checks, CPU tests).
"""
from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG_DIR, "csrc")
INCLUDE = os.path.join(os.path.dirname(PKG_DIR), "include")
LIB_NAME = "libdetkernels_b200.so"
LIB_PATH = os.path.join(PKG_DIR, LIB_NAME)
STAMP_PATH = LIB_PATH + ".srchash"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "--expt-relaxed-constexpr",
]


def _sources():
    files = []
    for d in (CSRC, INCLUDE):
        for name in sorted(os.listdir(d)):
            if name.endswith((".cu", ".cuh", ".h")):
                files.append(os.path.join(d, name))
    return files


def source_hash() -> str:
    h = hashlib.sha256()
    for path in _sources():
        h.update(os.path.basename(path).encode())
        with open(path, "rb") as f:
            h.update(f.read())
    h.update(" ".join(NVCC_FLAGS).encode())
    return h.hexdigest()


def nvcc_path() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the detkernels_b200 library needs the CUDA toolkit to build")


def is_up_to_date() -> bool:
    if not os.path.exists(LIB_PATH) or not os.path.exists(STAMP_PATH):
        return False
    with open(STAMP_PATH) as f:
        return f.read().strip() == source_hash()


def build(force: bool = False, verbose: bool = True) -> str:
    """Compile csrc/dk_lib.cu into LIB_PATH unless it is already current."""
    if not force and is_up_to_date():
        return LIB_PATH
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc_path(), *NVCC_FLAGS, "-I", INCLUDE, "-o", tmp, os.path.join(CSRC, "dk_lib.cu")]
    if verbose:
        print("[detkernels_b200] " + " ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("nvcc failed building %s" % LIB_NAME)
    os.replace(tmp, LIB_PATH)
    with open(STAMP_PATH, "w") as f:
        f.write(source_hash())
    return LIB_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv)
    print(LIB_PATH)
