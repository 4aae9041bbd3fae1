"""B-spline basis kernels on the GPU against the oracle (the reference's own PyTorch
Cox-de Boor, pinned by tests/golden/make_golden_bspline.py):
  - forward bit-identical to the fp32 reference recursion (same operation order) on every
    golden case — orders 1..5, uniform and adaptive grids, up to 59 knots — and on random
    inputs inside, at the edges of and outside the grid;
  - dL/dx within 1e-5 of the float64 autograd value relative to the sum of |terms|, and at
    the reference suite's bars (forward 1e-5, backward 1e-4, gradcheck in float64);
  - FusedKANLinear forward / backward against the reference KANLinear formulation;
  - non-finite inputs give NaN like the reference recursion;
  - a 16.7 M-element batch: sampled rows against the oracle and the partition of unity over
    the whole output."""

import json
import os

import numpy as np
import pytest
import torch

from oracle import bspline_oracle as bs
from rational_kat_cu_b200 import bspline as kb

pytestmark = pytest.mark.gpu

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
MANIFEST = json.load(open(os.path.join(HERE, "bspline_cases.json")))["cases"]


def golden(name):
    data = np.load(os.path.join(HERE, "golden_bspline.npz"))
    meta = next(c for c in MANIFEST if c["name"] == name)
    return meta, {k: torch.from_numpy(data[f"{name}/{k}"]) for k in ("x", "grid", "bases", "gb", "dx")}


def dx_term_scale(x, grid, order, gb):
    """Float64 sum over j of |grad_j * dB_j/dx| per element (tolerance scale)."""
    xd = x.detach().double().requires_grad_(True)
    bases = bs.b_splines(xd, grid.double(), order)
    scale = torch.zeros_like(xd)
    for j in range(bases.shape[-1]):
        g, = torch.autograd.grad(bases[..., j].sum(), xd, retain_graph=True)
        scale += (gb[..., j].double() * g).abs()
    return scale


def check_dx(dx, x, grid, order, gb, name, rtol=1e-5):
    _, dx64 = bs.b_splines_fwd_bwd(x, grid, order, gb, compute_dtype=torch.float64)
    scale = dx_term_scale(x, grid, order, gb)
    err = (dx.double() - dx64).abs()
    bad = err > rtol * scale + 1e-30
    assert not bool(bad.any()), f"{name}: {int(bad.sum())} dx values out of tolerance"


@pytest.mark.parametrize("name", [c["name"] for c in MANIFEST])
def test_golden_cases(name, cuda_device):
    meta, c = golden(name)
    order = meta["order"]
    x = c["x"].to(cuda_device)
    grid = c["grid"].to(cuda_device)
    bases = kb.bspline_basis_fwd(x, grid, order).cpu()
    assert bases.shape == c["bases"].shape
    assert torch.equal(bases, c["bases"]), name
    dx = kb.bspline_basis_bwd(x, grid, c["gb"].to(cuda_device), order).cpu()
    check_dx(dx, c["x"], c["grid"], order, c["gb"], name)
    assert (dx - c["dx"]).abs().max().item() < 1e-4 * max(1.0, c["dx"].abs().max().item())


@pytest.mark.parametrize("B,D,grid_size,order", [
    (4, 32, 8, 3), (16, 128, 8, 3), (1, 64, 8, 3), (4, 32, 5, 3), (4, 64, 3, 2),
    (257, 33, 7, 1), (64, 100, 10, 4), (9, 17, 30, 5),
    # cubic grid 8 / grid 5 (the kernels with the knot count compiled in, 32-row tiles):
    # batches that end inside a warp's rows, ragged feature columns, several column tiles
    (37, 45, 8, 3), (33, 70, 5, 3), (70, 64, 8, 3), (5, 96, 5, 3), (129, 31, 8, 3),
])
def test_random_inputs(B, D, grid_size, order, cuda_device):
    g = torch.Generator().manual_seed(B * D + order)
    x = torch.randn(B, D, generator=g) * 1.3
    x[0, : min(D, 4)] = torch.tensor([-1.0, 1.0, 0.0, 5.0])[: min(D, 4)]   # knots and outside
    grid = bs.make_grid(D, grid_size, order)
    gb = torch.randn(B, D, grid_size + order, generator=g)
    ref, _ = bs.b_splines_fwd_bwd(x, grid, order, gb)
    out = kb.bspline_basis_fwd(x.to(cuda_device), grid.to(cuda_device), order).cpu()
    assert torch.equal(out, ref)
    assert (out - ref).abs().max().item() < 1e-5          # the reference suite's forward bar
    dx = kb.bspline_basis_bwd(x.to(cuda_device), grid.to(cuda_device), gb.to(cuda_device),
                              order).cpu()
    check_dx(dx, x, grid, order, gb, f"random {B}x{D}")


def test_backward_matches_autograd_reference_bar(cuda_device):
    torch.manual_seed(42)
    B, D = 8, 64
    grid = bs.make_grid(D)
    x = torch.randn(B, D)
    gb = torch.randn(B, D, 11)
    _, dx_ref = bs.b_splines_fwd_bwd(x, grid, 3, gb)
    x_dev = x.to(cuda_device).requires_grad_(True)
    kb.BSplineBasis.apply(x_dev, grid.to(cuda_device), 3).backward(gb.to(cuda_device))
    assert (x_dev.grad.cpu() - dx_ref).abs().max().item() < 1e-4


def test_gradcheck(cuda_device):
    torch.manual_seed(42)
    B, D = 4, 32
    grid = bs.make_grid(D).to(cuda_device)
    x = torch.randn(B, D, device=cuda_device, dtype=torch.float64, requires_grad=True)

    def fn(x):
        return kb.BSplineBasis.apply(x.float(), grid.float(), 3).to(torch.float64)

    assert torch.autograd.gradcheck(fn, (x,), eps=1e-4, atol=1e-3, rtol=1e-3)


def test_non_finite_and_outside(cuda_device):
    grid = bs.make_grid(8, 8, 3)
    x = torch.tensor([[float("nan"), float("inf"), -float("inf"), -5.0, 5.0, -1.75, 1.749,
                       0.0]])
    ref = bs.b_splines(x, grid, 3)
    out = kb.bspline_basis_fwd(x.to(cuda_device), grid.to(cuda_device), 3).cpu()
    assert torch.equal(torch.isnan(out), torch.isnan(ref))
    fin = ~torch.isnan(ref)
    assert torch.equal(out[fin], ref[fin])
    gb = torch.ones(1, 8, 11)
    dx = kb.bspline_basis_bwd(x.to(cuda_device), grid.to(cuda_device), gb.to(cuda_device), 3).cpu()
    assert torch.isnan(dx[0, :3]).all() and dx[0, 3] == 0 and dx[0, 4] == 0


def test_fused_kan_linear_matches_reference(cuda_device):
    torch.manual_seed(42)
    B, D, O = 4, 64, 48
    layer = kb.FusedKANLinear(D, O, grid_size=8).to(cuda_device)
    assert torch.equal(layer.grid.cpu(), bs.make_grid(D, 8, 3))
    x = torch.randn(B, D, device=cuda_device, requires_grad=True)
    y = layer(x)
    assert y.shape == (B, O)
    xr = x.detach().clone().requires_grad_(True)
    bw = layer.base_weight.detach().clone().requires_grad_(True)
    sw = layer.spline_weight.detach().clone().requires_grad_(True)
    yr = bs.kan_linear(xr, layer.grid, 3, bw, sw)
    assert (y - yr).abs().max().item() < 1e-5
    gy = torch.randn_like(y)
    y.backward(gy)
    yr.backward(gy)
    for name, a, b in (("dx", x.grad, xr.grad), ("base_w", layer.base_weight.grad, bw.grad),
                       ("spline_w", layer.spline_weight.grad, sw.grad)):
        assert (a - b).abs().max().item() < 1e-4 * max(1.0, b.abs().max().item()), name


def test_update_grid(cuda_device):
    torch.manual_seed(3)
    layer = kb.FusedKANLinear(16, 8, grid_size=5).to(cuda_device)
    x = torch.randn(64, 16, device=cuda_device) * 2
    layer.update_grid(x)
    g = layer.grid
    assert g.shape == (16, 5 + 2 * 3 + 1)
    assert bool((g[:, 1:] >= g[:, :-1]).all())
    assert bool((g[:, 3] <= x.min(0)[0]).all()) and bool((g[:, -4] >= x.max(0)[0]).all())
    out = kb.bspline_basis_fwd(x, g, 3).cpu()
    assert torch.equal(out, bs.b_splines(x.cpu(), g.cpu(), 3))


def test_large_batch(cuda_device):
    B, D, gs, order = 16384, 1024, 8, 3
    gen = torch.Generator(device=cuda_device).manual_seed(0)
    x = torch.randn(B, D, generator=gen, device=cuda_device) * 0.6
    grid = bs.make_grid(D, gs, order).to(cuda_device)
    bases = kb.bspline_basis_fwd(x, grid, order)
    rows = torch.cat([torch.arange(0, 64), torch.arange(B - 64, B)])
    ref = bs.b_splines(x[rows].cpu(), grid.cpu(), order)
    assert torch.equal(bases[rows].cpu(), ref)
    inside = (x >= grid[:, order]) & (x < grid[:, -1 - order])
    s = bases.sum(-1)
    assert bool(((s - 1.0).abs()[inside] < 1e-5).all())
    assert bool((s[~inside] < 1.0 + 1e-5).all())
