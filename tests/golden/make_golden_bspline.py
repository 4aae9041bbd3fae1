"""Generate golden_bspline.npz / bspline_cases.json by running the REFERENCE's own PyTorch
B-spline basis.

The reference package rational_kat_cu defines the Cox-de Boor basis it fuses in PyTorch in its
test suite (tests/test_bspline.py: _ref_b_splines :11-24 and the grid builder _make_grid
:27-33).  This script takes those two functions from the reference's source file (only those:
the module's imports pull in Triton launchers that need a GPU), runs them on seeded CPU inputs
in fp32 with torch autograd for dL/dx, and stores x, grid, bases, grad_bases and dx.

Usage (needs the reference checkout; the fixtures are committed):
  python tests/golden/make_golden_bspline.py /path/to/rational_kat_cu   (or set KAT_REFERENCE_ROOT)
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
        sys.exit("usage: python tests/golden/make_golden_bspline.py /path/to/rational_kat_cu "
                 "(or set KAT_REFERENCE_ROOT)")
    return root


def load_functions(ref_root: str):
    path = os.path.join(ref_root, "tests", "test_bspline.py")
    tree = ast.parse(open(path).read(), filename=path)
    want = {"_ref_b_splines", "_make_grid"}
    body = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name in want]
    assert {n.name for n in body} == want, "reference functions not found"
    ns = {"torch": torch}
    exec(compile(ast.Module(body=body, type_ignores=[]), path, "exec"), ns)
    return ns["_ref_b_splines"], ns["_make_grid"]


CASES = [
    # name, B, D, grid_size, order, seed, x scale, grid kind
    ("b4_d32_g8_o3", 4, 32, 8, 3, 42, 1.0, "uniform"),
    ("b16_d128_g8_o3", 16, 128, 8, 3, 43, 1.0, "uniform"),
    ("b1_d64_g8_o3", 1, 64, 8, 3, 44, 1.0, "uniform"),
    ("b4_d32_g5_o3", 4, 32, 5, 3, 45, 1.0, "uniform"),
    ("b4_d64_g3_o2", 4, 64, 3, 2, 46, 1.0, "uniform"),
    ("b8_d48_g5_o1", 8, 48, 5, 1, 47, 1.0, "uniform"),
    ("b8_d24_g12_o4", 8, 24, 12, 4, 48, 1.2, "uniform"),
    ("b6_d40_g20_o5", 6, 40, 20, 5, 49, 1.2, "uniform"),
    ("b16_d32_g8_o3_wide", 16, 32, 8, 3, 50, 3.0, "uniform"),
    ("b32_d16_g8_o3_adaptive", 32, 16, 8, 3, 51, 1.0, "adaptive"),
    ("b8_d16_g52_o3_many_knots", 8, 16, 52, 3, 52, 1.0, "uniform"),
]


def adaptive_grid(x, grid_size, order, margin=0.01):
    """Per-feature quantile knots (efficient-KAN's update_grid rule) from x."""
    xs = x.sort(dim=0)[0]
    pos = torch.linspace(0, x.shape[0] - 1, grid_size + 1, dtype=torch.long)
    g = xs[pos].t()
    step = (g[:, -1] - g[:, 0]) / grid_size
    left = g[:, :1] - step.unsqueeze(1) * torch.arange(order, 0, -1)
    right = g[:, -1:] + step.unsqueeze(1) * torch.arange(1, order + 1)
    return torch.cat([left - margin * step.unsqueeze(1), g,
                      right + margin * step.unsqueeze(1)], dim=1).contiguous()


def main():
    ref_root = reference_root()
    ref_b_splines, ref_make_grid = load_functions(ref_root)
    arrays, manifest = {}, []
    for name, B, D, gs, order, seed, xs, kind in CASES:
        gen = torch.Generator().manual_seed(seed)
        x = torch.randn(B, D, generator=gen) * xs
        if kind == "adaptive":
            grid = adaptive_grid(x, gs, order)
        else:
            grid = ref_make_grid(D, gs, order, device="cpu")
        xr = x.clone().requires_grad_(True)
        bases = ref_b_splines(xr, grid, order)
        gb = torch.randn(bases.shape, generator=gen)
        bases.backward(gb)
        for key, val in (("x", x), ("grid", grid), ("bases", bases.detach()), ("gb", gb),
                         ("dx", xr.grad)):
            arrays[f"{name}/{key}"] = val.numpy().astype(np.float32)
        manifest.append({"name": name, "B": B, "D": D, "grid_size": gs, "order": order,
                         "seed": seed, "x_scale": xs, "grid": kind,
                         "n_knots": gs + 2 * order + 1})
    np.savez_compressed(os.path.join(HERE, "golden_bspline.npz"), **arrays)
    with open(os.path.join(HERE, "bspline_cases.json"), "w") as fh:
        json.dump({"source": "reference tests/test_bspline.py:11-33 (_ref_b_splines, "
                             f"_make_grid), torch {torch.__version__}, CPU fp32, autograd",
                   "cases": manifest}, fh, indent=1)
    print(f"wrote {len(manifest)} cases")


if __name__ == "__main__":
    main()
