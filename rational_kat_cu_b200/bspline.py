"""B-spline basis evaluation (Cox-de Boor) and the KAN linear layer built on it.

Drop-in for the reference's rational_kat_cu/bspline_basis.py:
  bspline_basis_fwd(x, grid, spline_order)              <- :262-296
  bspline_basis_bwd(x, grid, grad_basis, spline_order)  <- :562-599
  BSplineBasis (autograd Function)                      <- :602-619
  FusedKANLinear (efficient-KAN's KANLinear API)        <- :624-687
The basis runs on the sm_100a kernels of libkat_rational.so (kat_bspline_basis_fwd / _bwd,
include/kat_bspline.h): one thread per input element evaluates only the spline orders'
non-zero triangle on its knot span, with the reference's operation order, so the forward
matches the reference's PyTorch recursion bit for bit.  The grid (knots) is
[in_features, n_knots] fp32, non-decreasing along each row; x is [batch, in_features] fp32.
Unlike the reference's unrolled kernel (n_knots <= 15, spline order 3), any order 1..5 and up
to 64 knots are accepted.
"""

from __future__ import annotations

import ctypes

import torch
from torch import Tensor

from . import _native


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _check(x: Tensor, grid: Tensor, spline_order: int):
    if not (x.is_cuda and grid.is_cuda):
        raise RuntimeError("bspline_basis: x and grid must be CUDA tensors; there is no CPU "
                           "implementation")
    if x.dim() != 2 or grid.dim() != 2 or grid.shape[0] != x.shape[1]:
        raise ValueError(f"bspline_basis: expected x [B, D] and grid [D, n_knots], got "
                         f"{tuple(x.shape)} and {tuple(grid.shape)}")
    n_knots = grid.shape[1]
    if not 1 <= spline_order <= 5 or not spline_order + 2 <= n_knots <= 64:
        raise ValueError(f"bspline_basis: spline_order must be 1..5 and n_knots in "
                         f"[spline_order + 2, 64], got {spline_order} and {n_knots}")
    return n_knots, n_knots - 1 - spline_order


def bspline_basis_fwd(x: Tensor, grid: Tensor, spline_order: int = 3) -> Tensor:
    """bases [B, D, n_basis] (fp32) of x [B, D] on grid [D, n_knots]."""
    n_knots, n_basis = _check(x, grid, spline_order)
    B, D = x.shape
    xf = x.detach().float().contiguous()
    gf = grid.detach().float().contiguous()
    out = torch.empty(B, D, n_basis, device=x.device, dtype=torch.float32)
    with torch.cuda.device(x.device):
        st = _native.lib().kat_bspline_basis_fwd(xf.data_ptr(), gf.data_ptr(), out.data_ptr(),
                                                 B, D, n_knots, spline_order, _stream(x.device))
    _native.check("kat_bspline_basis_fwd", st)
    return out


def bspline_basis_bwd(x: Tensor, grid: Tensor, grad_basis: Tensor,
                      spline_order: int = 3) -> Tensor:
    """dL/dx [B, D] (fp32) from dL/dbases [B, D, n_basis]."""
    n_knots, n_basis = _check(x, grid, spline_order)
    B, D = x.shape
    if tuple(grad_basis.shape) != (B, D, n_basis):
        raise ValueError(f"bspline_basis: grad_basis shape {tuple(grad_basis.shape)} != "
                         f"{(B, D, n_basis)}")
    xf = x.detach().float().contiguous()
    gf = grid.detach().float().contiguous()
    gb = grad_basis.detach().float().contiguous()
    dx = torch.empty(B, D, device=x.device, dtype=torch.float32)
    with torch.cuda.device(x.device):
        st = _native.lib().kat_bspline_basis_bwd(xf.data_ptr(), gf.data_ptr(), gb.data_ptr(),
                                                 dx.data_ptr(), B, D, n_knots, spline_order,
                                                 _stream(x.device))
    _native.check("kat_bspline_basis_bwd", st)
    return dx


class BSplineBasis(torch.autograd.Function):
    """Fused B-spline basis evaluation; the grid gets no gradient (as in the reference)."""

    @staticmethod
    def forward(ctx, x: Tensor, grid: Tensor, spline_order: int = 3) -> Tensor:
        bases = bspline_basis_fwd(x, grid, spline_order)
        ctx.save_for_backward(x, grid)
        ctx.spline_order = spline_order
        return bases

    @staticmethod
    def backward(ctx, grad_basis: Tensor):
        x, grid = ctx.saved_tensors
        dx = bspline_basis_bwd(x, grid, grad_basis, ctx.spline_order)
        return dx.to(x.dtype), None, None


class FusedKANLinear(torch.nn.Module):
    """KAN linear layer (efficient-KAN's KANLinear API) on the fused basis kernels:
    y = base_activation(x) @ base_weight^T + einsum('bik,oik->bo', bases(x), spline_weight).
    The spline term is one GEMM of the [B, D * n_basis] basis matrix with the flattened
    spline weights."""

    def __init__(self, in_features: int, out_features: int, grid_size: int = 5,
                 spline_order: int = 3, grid_range=(-1.0, 1.0), base_activation=None):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.grid_size = grid_size
        self.spline_order = spline_order
        self.n_basis = grid_size + spline_order
        self.base_activation = base_activation or torch.nn.SiLU()
        self.base_weight = torch.nn.Parameter(torch.empty(out_features, in_features))
        self.spline_weight = torch.nn.Parameter(
            torch.empty(out_features, in_features, self.n_basis))
        # uniform knots on grid_range, extended by spline_order steps on each side (the
        # same arithmetic as the reference, bspline_basis.py:645-651, so the grids are equal)
        inner = torch.linspace(grid_range[0], grid_range[1], grid_size + 1)
        h = (grid_range[1] - grid_range[0]) / grid_size
        left = inner[0] - h * torch.arange(spline_order, 0, -1)
        right = inner[-1] + h * torch.arange(1, spline_order + 1)
        knots = torch.cat([left, inner, right])
        self.register_buffer("grid", knots.unsqueeze(0).expand(in_features, -1).clone())
        self.reset_parameters()

    def reset_parameters(self) -> None:
        torch.nn.init.kaiming_uniform_(self.base_weight, a=5 ** 0.5)
        torch.nn.init.kaiming_uniform_(self.spline_weight, a=5 ** 0.5)

    def b_splines(self, x: Tensor) -> Tensor:
        return BSplineBasis.apply(x, self.grid, self.spline_order)

    @torch.no_grad()
    def update_grid(self, x: Tensor, margin: float = 0.01) -> None:
        """Knots from the batch's per-feature quantiles (grid_size + 1 of them, evenly spaced
        in sorted order), extended by spline_order uniform steps and a margin on each side."""
        batch = x.shape[0]
        xs = x.sort(dim=0)[0]
        pos = torch.linspace(0, batch - 1, self.grid_size + 1, device=x.device,
                             dtype=torch.long)
        adaptive = xs[pos].t()
        step = (adaptive[:, -1] - adaptive[:, 0]) / self.grid_size
        k = self.spline_order
        left = adaptive[:, :1] - step.unsqueeze(1) * torch.arange(k, 0, -1, device=x.device)
        right = adaptive[:, -1:] + step.unsqueeze(1) * torch.arange(1, k + 1, device=x.device)
        left = left - margin * step.unsqueeze(1)
        right = right + margin * step.unsqueeze(1)
        self.grid.copy_(torch.cat([left, adaptive, right], dim=1))

    def forward(self, x: Tensor) -> Tensor:
        base = torch.nn.functional.linear(self.base_activation(x), self.base_weight)
        bases = self.b_splines(x)
        spline = bases.reshape(x.shape[0], -1) @ self.spline_weight.reshape(
            self.out_features, -1).t()
        return base + spline

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"grid_size={self.grid_size}, spline_order={self.spline_order}")
