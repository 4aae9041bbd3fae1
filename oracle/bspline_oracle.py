"""ORACLE — test infrastructure only.  Only tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline leg may import this module; the library never does.

A restatement, in PyTorch, of the reference's B-spline basis (rational_kat_cu of
felippe-alves/rational_kat_cu):

  b_splines      <- the reference's PyTorch Cox-de Boor, tests/test_bspline.py:11-24
                    (the recursion of efficient-KAN's KANLinear.b_splines): order-0
                    indicators t_i <= x < t_{i+1}; level k from ((x - t_i) / clamp(t_{i+k} -
                    t_i, 1e-8)) * B_i + ((t_{i+k+1} - x) / clamp(t_{i+k+1} - t_{i+1}, 1e-8)) *
                    B_{i+1}; gradients by torch autograd
  make_grid      <- tests/test_bspline.py:27-33 (uniform knots on [-1, 1] extended by
                    spline_order steps each side, one row per feature)
  kan_linear     <- tests/test_bspline.py:36-65 (_RefKANLinear.forward): SiLU base branch
                    plus the einsum of the bases with the spline weights

`compute_dtype=torch.float64` gives the float64 restatement.
"""

from __future__ import annotations

import torch


def b_splines(x: torch.Tensor, grid: torch.Tensor, spline_order: int) -> torch.Tensor:
    """bases [B, D, n_knots - 1 - spline_order] of x [B, D] on grid [D, n_knots]."""
    xe = x.unsqueeze(-1)
    bases = ((xe >= grid[:, :-1]) & (xe < grid[:, 1:])).to(x.dtype)
    for k in range(1, spline_order + 1):
        n = bases.shape[-1]
        t_lo, t_hi = grid[:, :n - 1], grid[:, k:n - 1 + k]
        t_lo1, t_hi1 = grid[:, 1:n], grid[:, k + 1:n + k]
        left = (xe - t_lo) / (t_hi - t_lo).clamp(min=1e-8) * bases[..., :-1]
        right = (t_hi1 - xe) / (t_hi1 - t_lo1).clamp(min=1e-8) * bases[..., 1:]
        bases = left + right
    return bases.contiguous()


def b_splines_fwd_bwd(x: torch.Tensor, grid: torch.Tensor, spline_order: int,
                      grad_bases: torch.Tensor, compute_dtype: torch.dtype = torch.float32):
    """bases and dL/dx (autograd) in `compute_dtype`."""
    xc = x.detach().to(compute_dtype).requires_grad_(True)
    bases = b_splines(xc, grid.detach().to(compute_dtype), spline_order)
    bases.backward(grad_bases.detach().to(compute_dtype))
    return bases.detach(), xc.grad


def make_grid(features: int, grid_size: int = 8, spline_order: int = 3) -> torch.Tensor:
    step = 2.0 / grid_size
    uniform = torch.linspace(-1, 1, grid_size + 1)
    left = uniform[0] - step * torch.arange(spline_order, 0, -1)
    right = uniform[-1] + step * torch.arange(1, spline_order + 1)
    return torch.cat([left, uniform, right]).unsqueeze(0).expand(features, -1).clone()


def kan_linear(x, grid, spline_order, base_weight, spline_weight):
    base = torch.nn.functional.linear(torch.nn.functional.silu(x), base_weight)
    spline = torch.einsum("bik,oik->bo", b_splines(x, grid, spline_order), spline_weight)
    return base + spline
