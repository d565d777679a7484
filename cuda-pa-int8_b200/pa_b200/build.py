"""Build libpa_b200.so (the C-ABI CUDA library) in-tree with nvcc for sm_100a.

The library has no torch dependency: nvcc compiles csrc/*.cu into one shared object that
exports the functions declared in include/pa_b200.h. It is rebuilt only when a source or
header is newer than the library.
"""

import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT_DIR = os.path.dirname(PKG_DIR)               # cuda-pa-int8_b200/
REPO_DIR = os.path.dirname(ROOT_DIR)              # repository root
CSRC_DIR = os.path.join(ROOT_DIR, "csrc")
INCLUDE_DIR = os.path.join(REPO_DIR, "include")
LIB_NAME = "libpa_b200.so"
LIB_PATH = os.path.join(PKG_DIR, LIB_NAME)

SOURCES = ["decode.cu", "quant.cu", "capi.cu", "noalloc.cu"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + [
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-O3",
    "-shared",
]


def nvcc_path():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libpa_b200.so")


def _inputs():
    files = [os.path.join(CSRC_DIR, s) for s in SOURCES]
    for d in (CSRC_DIR, INCLUDE_DIR):
        for f in os.listdir(d):
            if f.endswith((".h", ".cuh")):
                files.append(os.path.join(d, f))
    return files


def needs_build():
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    return any(os.path.getmtime(f) > t for f in _inputs())


def build(force=False, verbose=False):
    """Compile the library if it is missing or stale; return its path."""
    if not force and not needs_build():
        return LIB_PATH
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc_path()] + NVCC_FLAGS + ["-I", INCLUDE_DIR, "-I", CSRC_DIR, "-o", tmp]
    cmd += [os.path.join(CSRC_DIR, s) for s in SOURCES]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + res.stdout + res.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
