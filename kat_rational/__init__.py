"""Import-name shim: `from kat_rational import KAT_Group` keeps working for callers of the
reference package (kat_rational/__init__.py:1-4); everything lives in rational_kat_cu_b200."""

from rational_kat_cu_b200 import (  # noqa: F401
    KAT_Group,
    KAT_Group2D,
    KAT_Group_Torch,
    RationalTriton1DGroup,
    RationalTriton2D,
)
