"""Build recipe for libkat_rational.so (the sm_100a kernels behind the C ABI).

`build()` runs nvcc on csrc/kat_rational.cu, csrc/kat_bspline.cu and csrc/kat_gemm.cu for
`-gencode arch=compute_100a,code=sm_100a` and writes the shared library next to this file, so
it travels with the source tree.  It rebuilds only when a source or a public header is newer
than the library.  `build(debug=True)` writes libkat_rational_debug.so from the same sources
with -DKAT_DEBUG_BOUNDS=1: every global access, workspace slot and plan invariant of the
activation kernels is checked, and a violation sets KAT_DEVICE_BOUNDS in the device status
word instead of being made (the GPU-side stand-in for compute-sanitizer; tests only).
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
SOURCES = [os.path.join(PKG_DIR, "csrc", "kat_rational.cu"),
           os.path.join(PKG_DIR, "csrc", "kat_bspline.cu"),
           os.path.join(PKG_DIR, "csrc", "kat_gemm.cu")]
HEADERS = [os.path.join(REPO_DIR, "include", "kat_rational.h"),
           os.path.join(REPO_DIR, "include", "kat_bspline.h"),
           os.path.join(REPO_DIR, "include", "kat_gemm.h"),
           os.path.join(PKG_DIR, "csrc", "kat_math.cuh"),
           os.path.join(PKG_DIR, "csrc", "kat_plan.h")]
LIBRARY = os.path.join(PKG_DIR, "libkat_rational.so")
DEBUG_LIBRARY = os.path.join(PKG_DIR, "libkat_rational_debug.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-O2",
    "-shared",
    "-diag-suppress", "177",
]


def find_nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def is_stale(target: str = LIBRARY) -> bool:
    if not os.path.exists(target):
        return True
    lib_t = os.path.getmtime(target)
    return any(os.path.getmtime(p) > lib_t for p in (*SOURCES, *HEADERS, __file__))


def build(force: bool = False, verbose: bool = False, debug: bool = False) -> str:
    """Compile the library (or its bounds-checked debug build) if needed; return its path."""
    target = DEBUG_LIBRARY if debug else LIBRARY
    if not force and not is_stale(target):
        return target
    cmd = [find_nvcc(), *NVCC_FLAGS, "-I", os.path.join(REPO_DIR, "include"),
           *(["-DKAT_DEBUG_BOUNDS=1"] if debug else []), "-o", target + ".tmp", *SOURCES]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose:
        print(res.stderr, file=sys.stderr)
    os.replace(target + ".tmp", target)
    return target


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv,
                debug="--debug" in sys.argv))
