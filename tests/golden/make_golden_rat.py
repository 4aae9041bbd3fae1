"""Generate golden_rat.npz / rat_cases.json by running the REFERENCE's own definition of the
rat_cuda formula.

The reference package rational_kat_cu defines its abs-after-sum activation in PyTorch in
its test suite (tests/test_correctness.py:16-39, `_rat_ref`: Q = 1 + |b0 x + ... + b3 x^4|,
numerator a [6] shared by the groups).  This script takes that function from the reference's
source file (only that function: the module's imports pull in Triton launchers that need a
GPU), runs it on seeded CPU inputs in fp32 with torch autograd for the gradients, and stores
inputs, y, dx, d a [6] and d b [G, 4].

One convention differs between the reference's two implementations: at D(x) = 0, torch's
abs backward uses sgn(0) = 0 while the reference kernels (rat_cuda's actual backward,
rational_kat_cu/rational_bwd_triton.py:111) use +1.  Cases are generated with inputs where
D != 0 everywhere except the identity case (b = 0, D == 0 everywhere), whose d b is
recorded as not comparable ("db_comparable": false).

Usage (needs the reference checkout; the fixtures are committed):
  python tests/golden/make_golden_rat.py /path/to/rational_kat_cu   (or set KAT_REFERENCE_ROOT)
"""

from __future__ import annotations

import ast
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
def reference_root() -> str:
    """The reference checkout: the first command-line argument, else $KAT_REFERENCE_ROOT."""
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("KAT_REFERENCE_ROOT")
    if not root:
        sys.exit("usage: python tests/golden/make_golden_rat.py /path/to/rational_kat_cu "
                 "(or set KAT_REFERENCE_ROOT)")
    return root


def load_rat_ref(ref_root: str):
    path = os.path.join(ref_root, "tests", "test_correctness.py")
    tree = ast.parse(open(path).read(), filename=path)
    fn = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "_rat_ref"]
    assert len(fn) == 1, "reference _rat_ref not found"
    module = ast.Module(body=fn, type_ignores=[])
    ns = {"torch": torch}
    exec(compile(module, path, "exec"), ns)
    return ns["_rat_ref"]


CASES = [
    # name, N, D, G, seed, x_scale, coefficient kind, input dtype
    ("fwd_4x64_g8", 4, 64, 8, 42, 1.0, "randn", "f32"),
    ("fwd_32x256_g8", 32, 256, 8, 43, 1.0, "randn", "f32"),
    ("fwd_1x32_g4", 1, 32, 4, 44, 1.0, "randn", "f32"),
    ("bwd_32x256_g8", 32, 256, 8, 45, 1.0, "randn", "f32"),
    ("wide_x_16x96_g3", 16, 96, 3, 46, 2.5, "randn", "f32"),
    ("g1_8x128", 8, 128, 1, 47, 1.0, "randn", "f32"),
    ("g64_4x768", 4, 768, 64, 48, 1.0, "randn", "f32"),
    ("bf16_in_16x128_g8", 16, 128, 8, 49, 1.0, "randn", "bf16"),
    ("f16_in_8x64_g8", 8, 64, 8, 50, 1.0, "randn", "f16"),
    ("identity_8x128_g8", 8, 128, 8, 51, 1.0, "identity", "f32"),
]


def main():
    ref_root = reference_root()
    rat_ref = load_rat_ref(ref_root)
    arrays, manifest = {}, []
    for name, N, D, G, seed, xs, kind, dt in CASES:
        gen = torch.Generator().manual_seed(seed)
        x = torch.randn(N, D, generator=gen) * xs
        if dt == "bf16":
            x = x.to(torch.bfloat16).float()
        elif dt == "f16":
            x = x.to(torch.float16).float()
        gy = torch.randn(N, D, generator=gen)
        if kind == "identity":
            a = torch.zeros(6)
            a[1] = 1.0
            b = torch.zeros(G, 4)
        else:
            a = torch.randn(6, generator=gen)
            b = torch.randn(G, 4, generator=gen)
        xr = x.clone().requires_grad_(True)
        ar = a.clone().requires_grad_(True)
        br = b.clone().requires_grad_(True)
        y = rat_ref(xr, ar, br)
        y.backward(gy)
        with torch.no_grad():
            xg = x.reshape(-1, G, D // G)
            d = b[:, -1].view(1, G, 1)
            for i in range(2, -1, -1):
                d = b[:, i].view(1, G, 1) + xg * d
            zeros = int(((xg * d) == 0).sum())
        for key, val in (("x", x), ("gy", gy), ("a", a), ("b", b), ("y", y.detach()),
                         ("dx", xr.grad), ("da", ar.grad), ("db", br.grad)):
            arrays[f"{name}/{key}"] = val.numpy().astype(np.float32)
        manifest.append({"name": name, "N": N, "D": D, "G": G, "seed": seed, "x_scale": xs,
                         "coefficients": kind, "input_dtype": dt, "d_zero_count": zeros,
                         "db_comparable": zeros == 0})
    np.savez_compressed(os.path.join(HERE, "golden_rat.npz"), **arrays)
    with open(os.path.join(HERE, "rat_cases.json"), "w") as fh:
        json.dump({"source": "reference tests/test_correctness.py:16-39 (_rat_ref), torch "
                             f"{torch.__version__}, CPU fp32, autograd",
                   "cases": manifest}, fh, indent=1)
    print(f"wrote {len(manifest)} cases")


if __name__ == "__main__":
    main()
