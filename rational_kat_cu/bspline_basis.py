"""Import-name shim for the reference module rational_kat_cu/bspline_basis.py: the fused
B-spline basis and FusedKANLinear, implemented in rational_kat_cu_b200.bspline."""

from rational_kat_cu_b200.bspline import (  # noqa: F401
    BSplineBasis,
    FusedKANLinear,
    bspline_basis_bwd,
    bspline_basis_fwd,
)
