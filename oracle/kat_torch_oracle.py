"""ORACLE — test infrastructure only.  Only tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline leg may import this module; the library never does.

A CPU restatement, in PyTorch, of the reference's group-rational path
(kat_rational/kat_1dgroup_torch.py of felippe-alves/rational_kat_cu), keeping its exact
sequence of tensor operations so that on the same machine it reproduces the reference's
fp32 results bit for bit:

  rational_1dgroup          <- Rational_CUDA_A_1DGroup, kat_1dgroup_torch.py:27-78
    group-major copy          :53-54   view [B,L,G,Dg] -> permute(2,0,1,3) -> [G, N/G]
    power stack               :7-24    [1, z, z*z, (z*z)*z, ...] stacked on dim 1
    numerator                 :60      bmm(w_num[G,1,6], powers)
    denominator               :63-69   bmm(|[1, w_den, 0-pad]|[G,1,6], powers)
    quotient, layout back     :72-76
  module forward            <- KAT_Group_Torch.forward, kat_1dgroup_torch.py:130-145
                               (numerator [1,6] repeated per group; gradients by autograd)
  2-D input [B, C]          -> viewed as [1, B, C] (the reference function needs 3-D input)
  NCHW input [B, C, H, W]   -> permuted to [B, H*W, C], evaluated, permuted back (the
                               reference has no CPU path for KAT_Group2D,
                               kat_rational/kat_2dgroup_triton.py:31)
  bf16 / fp16 input         -> upcast to fp32 (the reference's bmm rejects mixed dtypes),
                               evaluated, and rounded by the caller if it wants that dtype.

`compute_dtype=torch.float64` gives the float64 restatement of the same formula.
"""

from __future__ import annotations

import torch


def power_stack(z: torch.Tensor, n_num: int, n_den: int) -> torch.Tensor:
    """[G, n, M] stack of z**0 .. z**(n-1), n = max(n_num, n_den); kat_1dgroup_torch.py:7-24."""
    powers = [z]
    for _ in range(max(n_num, n_den) - 2):
        powers.append(powers[-1] * z)
    powers.insert(0, torch.ones_like(z))
    return torch.stack(powers, dim=1)


def rational_1dgroup(x: torch.Tensor, w_num: torch.Tensor, w_den: torch.Tensor,
                     group: int) -> torch.Tensor:
    """y = P/Q on x [B, L, D] with w_num [group, 6], w_den [group, 4] (kat_1dgroup_torch.py:27-78)."""
    B, L, D = x.shape
    n_num, n_den = w_num.size(1), w_den.size(1)
    per = D // group
    z = x.view(B, L, group, per).permute(2, 0, 1, 3).contiguous().view(group, B * L * per)
    xps = power_stack(z, n_num, n_den)
    num = torch.bmm(w_num.unsqueeze(1), xps).squeeze(1)
    den_coef = torch.cat([
        torch.ones(group, 1, device=x.device, dtype=w_den.dtype),
        w_den,
        torch.zeros(group, max(0, n_num - n_den - 1), device=x.device, dtype=w_den.dtype),
    ], dim=1)
    den = torch.bmm(den_coef.abs().unsqueeze(1), xps).squeeze(1)
    out = num.div(den)
    return out.view(group, B, L, per).permute(1, 2, 0, 3).contiguous().view(B, L, D)


def _to_blc(x: torch.Tensor, layout: str) -> torch.Tensor:
    if layout == "blc":
        return x
    if layout == "bc":
        return x.view(1, *x.shape)
    if layout == "nchw":
        B, C, H, W = x.shape
        return x.permute(0, 2, 3, 1).reshape(B, H * W, C)
    raise ValueError(layout)


def _from_blc(y: torch.Tensor, layout: str, shape) -> torch.Tensor:
    if layout == "blc":
        return y
    if layout == "bc":
        return y.view(shape)
    if layout == "nchw":
        B, C, H, W = shape
        return y.view(B, H, W, C).permute(0, 3, 1, 2).contiguous()
    raise ValueError(layout)


def forward(x: torch.Tensor, w_num_1x6: torch.Tensor, w_den: torch.Tensor, group: int,
            layout: str = "blc", compute_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Module-level forward (numerator [1, 6] repeated per group), no autograd."""
    with torch.no_grad():
        xc = x.to(compute_dtype)
        y = rational_1dgroup(_to_blc(xc, layout), w_num_1x6.to(compute_dtype).repeat(group, 1),
                             w_den.to(compute_dtype), group)
        return _from_blc(y, layout, x.shape)


def forward_backward(x: torch.Tensor, w_num_1x6: torch.Tensor, w_den: torch.Tensor, group: int,
                     grad_out: torch.Tensor, layout: str = "blc",
                     compute_dtype: torch.dtype = torch.float32):
    """y, dx, d w_num [1, 6], d w_den [group, 4] as torch autograd computes them for the
    reference module (KAT_Group_Torch.forward, kat_1dgroup_torch.py:130-145)."""
    xc = x.detach().to(compute_dtype).requires_grad_(True)
    wn = w_num_1x6.detach().to(compute_dtype).requires_grad_(True)
    wd = w_den.detach().to(compute_dtype).requires_grad_(True)
    y = rational_1dgroup(_to_blc(xc, layout), wn.repeat(group, 1), wd, group)
    y = _from_blc(y, layout, x.shape)
    y.backward(grad_out.detach().to(compute_dtype))
    return y.detach(), xc.grad, wn.grad, wd.grad
