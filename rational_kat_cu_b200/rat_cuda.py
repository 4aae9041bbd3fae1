"""rat_cuda: the grouped Padé activation with the abs-after-sum denominator.

Drop-in for the reference package `rational_kat_cu` (rational_kat_cu/__init__.py:5-51):

    y = P(x) / Q(x),  P(x) = a0 + a1 x + ... + a5 x^5          (numerator shared by all groups)
                      Q(x) = 1 + |b0 x + b1 x^2 + b2 x^3 + b3 x^4|  (raw b per group, abs after the sum)

`rat_cuda(x, a[6], b[G, 4])` expands the numerator to [G, 6] and calls
`_RationalGroupedFn.apply(x, a_grouped, b, G)`; the Function keeps the reference's
custom_fwd(cast_inputs=float32) / custom_bwd autocast behaviour and returns
(d_x, d_a_grouped[G, 6], d_b[G, 4], None), so autograd sums d_a over the groups for `a`.
The forward and backward run on the same sm_100a kernels as KAT_Group, selected with
KAT_FORMULA_ABS_SUM (kat_rational_fwd_formula / kat_rational_bwd_formula); the backward's
coefficient sums use the same fixed-order reduction, so they are reproducible run to run.
At D(x) = 0 the sign of D counts as +1, as in the reference kernels'
where(D < 0, -1, 1) (rational_kat_cu/rational_bwd_triton.py:111).

x is [N, D] (any leading shape is accepted and flattened; the channel dimension is last);
fp32, bf16 and fp16 run on the vectorised kernels; fp64 tensors (used by gradcheck) take the
float64 forward kernel and the fp32 backward, the precisions the reference kernels use for
them (its Triton forward computes in the input dtype, its backward in fp32).  Gradients of a
and b come back in the dtype of a and b.
"""

from __future__ import annotations

import torch
import torch.nn as nn
from torch import Tensor

from . import _native
from .rational_cuda import _bwd, _dims_1d, _fwd

FORMULA = _native.KAT_FORMULA_ABS_SUM


def rat_fwd_cuda(x: Tensor, a_grouped: Tensor, b: Tensor, g: int) -> Tensor:
    """Forward launcher (rational_kat_cu/__init__.py:29 -> kat_rational/rational_triton.py:76)."""
    return _fwd(x, a_grouped, b, g, _dims_1d(x, g), formula=FORMULA)


def rat_bwd_cuda(x: Tensor, a_grouped: Tensor, b: Tensor, grad_output: Tensor, g: int,
                 need_dx: bool = True):
    """Backward launcher with the argument order of rational_bwd_triton
    (rational_kat_cu/rational_bwd_triton.py:319-375): returns (dx, da[G, 6], db[G, 4])."""
    dx, da, db = _bwd(grad_output, x, a_grouped, b, g, _dims_1d(x, g), need_dx=need_dx,
                      formula=FORMULA)
    return dx, da.to(a_grouped.dtype), db.to(b.dtype)


class _RationalGroupedFn(torch.autograd.Function):
    """Grouped Padé rational activation, abs-after-sum denominator
    (rational_kat_cu/__init__.py:6-40)."""

    @staticmethod
    @torch.amp.custom_fwd(cast_inputs=torch.float32, device_type="cuda")
    def forward(ctx, x: Tensor, a_grouped: Tensor, b: Tensor, g: int) -> Tensor:
        ctx.save_for_backward(x, a_grouped, b)
        ctx.g = g
        return rat_fwd_cuda(x, a_grouped, b, g)

    @staticmethod
    @torch.amp.custom_bwd(device_type="cuda")
    def backward(ctx, grad_output: Tensor):
        x, a_grouped, b = ctx.saved_tensors
        d_x, d_a, d_b = rat_bwd_cuda(x, a_grouped, b, grad_output, ctx.g,
                                     need_dx=ctx.needs_input_grad[0])
        return d_x, d_a, d_b, None


def _rat_cuda_impl(x: Tensor, a: Tensor, b: Tensor) -> Tensor:
    g = b.shape[0]
    a_grouped = a.unsqueeze(0).expand(g, -1).contiguous()
    return _RationalGroupedFn.apply(x, a_grouped, b, g)


# Kept out of torch.compile tracing, as in the reference (rational_kat_cu/__init__.py:49-51).
rat_cuda = torch.compiler.disable(_rat_cuda_impl)


class RatGroup(nn.Module):
    """Module holding rat_cuda's coefficients: weight_numerator [6] (shared) and
    weight_denominator [num_groups, 4] (raw); forward(x) = rat_cuda(x, numerator,
    denominator).  The reference exposes only the function; the module is the same call with
    its parameters, for models and for the host-buffer pipeline."""

    formula = FORMULA

    def __init__(self, num_groups: int = 8, numerator=None, denominator=None):
        super().__init__()
        self.num_groups = num_groups
        a = torch.zeros(6) if numerator is None else torch.as_tensor(numerator, dtype=torch.float32)
        if numerator is None:
            a[1] = 1.0   # P(x) = x
        b = (torch.zeros(num_groups, 4) if denominator is None
             else torch.as_tensor(denominator, dtype=torch.float32).reshape(num_groups, 4))
        self.weight_numerator = nn.Parameter(a.reshape(6).clone())
        self.weight_denominator = nn.Parameter(b.clone())

    def forward(self, x: Tensor) -> Tensor:
        return rat_cuda(x, self.weight_numerator, self.weight_denominator)

    def extra_repr(self) -> str:
        return f"num_groups={self.num_groups}, formula=abs-after-sum"
