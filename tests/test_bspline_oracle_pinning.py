"""The B-spline oracle (oracle/bspline_oracle.py) pinned to the reference's own PyTorch
Cox-de Boor (tests/golden/make_golden_bspline.py ran the reference's _ref_b_splines and
_make_grid on these inputs), on the CPU: bases and dL/dx are reproduced bit for bit, the grid
builder gives the same knots, and the float64 restatement agrees within fp32 rounding."""

import json
import os

import numpy as np
import pytest
import torch

from oracle import bspline_oracle as bs

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
MANIFEST = json.load(open(os.path.join(HERE, "bspline_cases.json")))["cases"]
NAMES = [c["name"] for c in MANIFEST]


def case(name):
    data = np.load(os.path.join(HERE, "golden_bspline.npz"))
    meta = next(c for c in MANIFEST if c["name"] == name)
    return meta, {k: torch.from_numpy(data[f"{name}/{k}"]) for k in ("x", "grid", "bases", "gb", "dx")}


@pytest.mark.parametrize("name", NAMES)
def test_restatement_reproduces_reference(name):
    meta, c = case(name)
    bases, dx = bs.b_splines_fwd_bwd(c["x"], c["grid"], meta["order"], c["gb"])
    assert torch.equal(bases, c["bases"]), name
    assert torch.equal(dx, c["dx"]), name


@pytest.mark.parametrize("name", [n for n in NAMES if "adaptive" not in n])
def test_grid_builder(name):
    meta, c = case(name)
    assert torch.equal(bs.make_grid(meta["D"], meta["grid_size"], meta["order"]), c["grid"])


@pytest.mark.parametrize("name", NAMES)
def test_float64_restatement_agrees(name):
    meta, c = case(name)
    b64, dx64 = bs.b_splines_fwd_bwd(c["x"], c["grid"], meta["order"], c["gb"],
                                     compute_dtype=torch.float64)
    torch.testing.assert_close(c["bases"].double(), b64, rtol=0, atol=1e-6)
    scale = dx64.abs().max().item() + 1.0
    torch.testing.assert_close(c["dx"].double(), dx64, rtol=0, atol=1e-5 * scale)


def test_partition_of_unity_on_the_golden_cases():
    """Inside [t_p, t_{n-1-p}) the order-p basis sums to one."""
    for name in NAMES:
        meta, c = case(name)
        p, g = meta["order"], c["grid"]
        inside = (c["x"] >= g[:, p]) & (c["x"] < g[:, -1 - p])
        s = c["bases"].double().sum(-1)
        assert torch.allclose(s[inside], torch.ones_like(s[inside]), atol=1e-5), name
