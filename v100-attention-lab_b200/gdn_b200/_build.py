"""Build the sm_100a shared library ``libgdn_b200.so`` in place with nvcc.

The library is a plain C-ABI shared object (see include/gdn_b200.h); it links
the CUDA runtime statically and needs no framework at build or load time.
"""

from __future__ import annotations

import os
import shutil
import subprocess

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
SRC_DIR = os.path.join(os.path.dirname(PKG_DIR), "csrc")
INCLUDE_DIR = os.path.join(os.path.dirname(os.path.dirname(PKG_DIR)), "include")
LIB_PATH = os.path.join(PKG_DIR, "libgdn_b200.so")

SOURCES = ["gdn_fwd.cu", "gdn_wy_scan.cu", "gdn_noalloc.cu"]
HEADERS = ["tc.cuh", "tmap.h", "gdn_common.cuh", "gdn_wy_scan.h"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo",
    "-shared", "-Xcompiler", "-fPIC,-O2",
    "-Xptxas", "-warn-spills",
]


def nvcc_path() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build gdn_b200")


def _inputs():
    files = [os.path.join(SRC_DIR, f) for f in SOURCES + HEADERS]
    files.append(os.path.join(INCLUDE_DIR, "gdn_b200.h"))
    return files


def is_stale(lib_path: str = LIB_PATH) -> bool:
    if not os.path.exists(lib_path):
        return True
    mtime = os.path.getmtime(lib_path)
    return any(os.path.getmtime(f) > mtime for f in _inputs())


def build(force: bool = False, verbose: bool = False, lib_path: str = LIB_PATH) -> str:
    """Compile the library if it is missing or older than its sources."""
    if not force and not is_stale(lib_path):
        return lib_path
    tmp = lib_path + ".tmp"
    cmd = [nvcc_path(), *NVCC_FLAGS, "-I", INCLUDE_DIR, "-o", tmp,
           *[os.path.join(SRC_DIR, s) for s in SOURCES]]
    if verbose:
        print(" ".join(cmd))
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout, res.stderr)
    os.replace(tmp, lib_path)
    return lib_path


if __name__ == "__main__":
    print(build(force=True, verbose=True))
