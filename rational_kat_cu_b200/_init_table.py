"""Coefficient presets shipped in init.json (the reference's kat_rational/init.json, unchanged).

Each mode holds 6 numerator and 4 denominator coefficients fitted to a classic
activation; "ub"/"lb" (the fitting range) are carried but unused, as in the reference.
"""

from __future__ import annotations

import json
import os

INIT_JSON = os.path.join(os.path.dirname(os.path.abspath(__file__)), "init.json")


def load_table(path: str = INIT_JSON) -> dict:
    with open(path) as fh:
        return json.load(fh)


def modes() -> list:
    return list(load_table())
