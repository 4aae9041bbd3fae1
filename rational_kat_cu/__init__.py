"""Import-name shim: `from rational_kat_cu import rat_cuda` keeps working for callers of the
reference package (rational_kat_cu/__init__.py:1-51); the implementation lives in
rational_kat_cu_b200.rat_cuda; `rational_kat_cu.bspline_basis` maps to
rational_kat_cu_b200.bspline."""

from rational_kat_cu_b200.rat_cuda import (  # noqa: F401
    _RationalGroupedFn,
    rat_bwd_cuda as rational_bwd_triton,
    rat_cuda,
)
