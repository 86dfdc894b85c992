"""Builds the sm_100a shared library libfa_b200.so in this directory.

The reference JIT-compiles its extension with torch.utils.cpp_extension.load
on first import (fa_p100.py:21-28, -arch=sm_60). Here the library is a plain
C-ABI shared object compiled by nvcc for sm_100a only, built in-tree so it
travels with the source tree; `build()` is idempotent and skips the compile
when the library is newer than every source file.
"""
import os
import shutil
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIB_PATH = os.path.join(HERE, "libfa_b200.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo",
    "-Xcompiler", "-fPIC", "-shared",
]


def _sources():
    out = []
    for d in (CSRC, INCLUDE):
        for name in sorted(os.listdir(d)):
            if name.endswith((".cu", ".cuh", ".h")):
                out.append(os.path.join(d, name))
    return out


def _nvcc():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: cannot build libfa_b200.so")


def up_to_date():
    if not os.path.exists(LIB_PATH):
        return False
    lib_mtime = os.path.getmtime(LIB_PATH)
    return all(os.path.getmtime(s) <= lib_mtime for s in _sources())


def build(force=False, verbose=False):
    """Compile csrc/fa_b200.cu into libfa_b200.so (sm_100a). Returns its path."""
    if not force and up_to_date():
        return LIB_PATH
    tmp = LIB_PATH + ".tmp"
    cmd = [_nvcc(), *NVCC_FLAGS, "-o", tmp, os.path.join(CSRC, "fa_b200.cu")]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed building libfa_b200.so:\n" + res.stdout + res.stderr)
    if verbose:
        print(res.stdout + res.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force=True, verbose=True))
