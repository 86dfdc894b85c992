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
# The checked build: every TMA copy tests its coordinates and shared-memory
# alignment first (-DFAB_CHECK_TMA, fa_b200_debug_tma_check). Selected at load
# time by FA_B200_DEBUG=1; the release library is the default.
DEBUG_LIB_PATH = os.path.join(HERE, "libfa_b200_debug.so")

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


def checked_requested():
    """Whether FA_B200_DEBUG=1 asks for the checked library."""
    return os.environ.get("FA_B200_DEBUG", "0") == "1"


def lib_path(checked=None):
    if checked is None:
        checked = checked_requested()
    return DEBUG_LIB_PATH if checked else LIB_PATH


def up_to_date(checked=None):
    path = lib_path(checked)
    if not os.path.exists(path):
        return False
    lib_mtime = os.path.getmtime(path)
    return all(os.path.getmtime(s) <= lib_mtime for s in _sources())


def build(force=False, verbose=False, checked=None):
    """Compile csrc/fa_b200.cu into libfa_b200.so, or with checked (default:
    FA_B200_DEBUG=1) into libfa_b200_debug.so with -DFAB_CHECK_TMA (sm_100a
    either way). Returns the library's path."""
    if checked is None:
        checked = checked_requested()
    path = lib_path(checked)
    if not force and up_to_date(checked):
        return path
    tmp = path + ".tmp"
    cmd = [_nvcc(), *NVCC_FLAGS, *(["-DFAB_CHECK_TMA"] if checked else []), "-o", tmp,
           os.path.join(CSRC, "fa_b200.cu")]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed building {os.path.basename(path)}:\n" + res.stdout + res.stderr)
    if verbose:
        print(res.stdout + res.stderr)
    os.replace(tmp, path)
    return path


if __name__ == "__main__":
    print(build(force=True, verbose=True))
