"""__graft_entry__.smoke() on cuda:0: one KAT_Group (bf16 [2,197,768]) and one KAT_Group2D
(fp32 [2,64,14,14]) forward + backward through the modules, checked against the float64 C
restatement of the reference's formula."""

import os
import sys

import pytest

pytestmark = pytest.mark.gpu
sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def test_smoke():
    import __graft_entry__ as entry

    entry.smoke()
