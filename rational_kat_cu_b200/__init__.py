"""B200-native (sm_100a) group-rational activation for the Kolmogorov-Arnold Transformer.

Public API, matching the reference package `kat_rational` (kat_rational/__init__.py:1-4):
KAT_Group, KAT_Group2D, KAT_Group_Torch and the autograd Functions (also under their
reference names RationalTriton1DGroup / RationalTriton2D); and the reference package
`rational_kat_cu`'s front end rat_cuda (rational_kat_cu/__init__.py), the abs-after-sum
variant of the activation on the same kernels; and its B-spline basis kernels with the
FusedKANLinear layer (rational_kat_cu/bspline_basis.py).  `fused_gemm` holds the KAN block's
fc1 -> act2 -> fc2 with the activation inside tcgen05 GEMM epilogues (KANMlpFused).
"""

from . import fused_gemm
from .bspline import BSplineBasis, FusedKANLinear, bspline_basis_bwd, bspline_basis_fwd
from .fused_gemm import KANMlpFused, kan_mlp_fused
from .kat_1dgroup import KAT_Group
from .kat_1dgroup_torch import KAT_Group_Torch, Rational_CUDA_A_1DGroup
from .kat_2dgroup import KAT_Group2D
from .rat_cuda import RatGroup, rat_cuda
from .rational_cuda import (
    RationalCUDA1DGroup,
    RationalCUDA2D,
    RationalTriton1DGroup,
    RationalTriton2D,
    rational_bwd_cuda,
    rational_bwd_cuda_2d,
    rational_fwd_cuda,
    rational_fwd_cuda_2d,
)

__all__ = [
    "KAT_Group",
    "KAT_Group2D",
    "KAT_Group_Torch",
    "Rational_CUDA_A_1DGroup",
    "RationalCUDA1DGroup",
    "RationalCUDA2D",
    "RationalTriton1DGroup",
    "RationalTriton2D",
    "rational_fwd_cuda",
    "rational_bwd_cuda",
    "rational_fwd_cuda_2d",
    "rational_bwd_cuda_2d",
    "rat_cuda",
    "RatGroup",
    "BSplineBasis",
    "FusedKANLinear",
    "bspline_basis_fwd",
    "bspline_basis_bwd",
    "fused_gemm",
    "KANMlpFused",
    "kan_mlp_fused",
]
