"""ORACLE build recipe (test infrastructure): compiles kat_oracle.c into
oracle/_build/libkat_oracle.so with gcc (OpenMP when available).

The reference itself is not compiled here: its CPU path is PyTorch Python code
(kat_rational/kat_1dgroup_torch.py), restated in kat_torch_oracle.py, and its only C++
sources (src/*.cu, src/rational.cpp) are a torch CUDA extension for a different formula
that its own setup.py does not build.
"""

from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SOURCE = os.path.join(HERE, "kat_oracle.c")
OUT_DIR = os.path.join(HERE, "_build")
LIBRARY = os.path.join(OUT_DIR, "libkat_oracle.so")


def build(force: bool = False) -> str:
    if (not force and os.path.exists(LIBRARY)
            and os.path.getmtime(LIBRARY) >= max(os.path.getmtime(SOURCE),
                                                 os.path.getmtime(__file__))):
        return LIBRARY
    os.makedirs(OUT_DIR, exist_ok=True)
    base = ["gcc", "-O2", "-fPIC", "-shared", "-std=c11", "-o", LIBRARY + ".tmp", SOURCE, "-lm"]
    res = subprocess.run(base[:1] + ["-fopenmp"] + base[1:], capture_output=True, text=True)
    if res.returncode != 0:  # no OpenMP runtime: single-threaded build
        res = subprocess.run(base, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{res.stderr}")
    os.replace(LIBRARY + ".tmp", LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
