"""Loader for the committed golden vectors (made by tests/golden/make_golden.py from the
reference implementation)."""

from __future__ import annotations

import json
import os

import numpy as np
import torch

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TORCH_DTYPES = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}

_cache = {}


def manifest() -> list:
    with open(os.path.join(GOLDEN_DIR, "cases.json")) as fh:
        return json.load(fh)


def case_names() -> list:
    return [c["name"] for c in manifest()]


def load_case(name: str) -> dict:
    if "small" not in _cache:
        _cache["small"] = dict(np.load(os.path.join(GOLDEN_DIR, "golden_small.npz")))
    arr = _cache["small"]
    meta = next(c for c in manifest() if c["name"] == name)
    out = dict(meta)
    for key in ("x", "grad_out", "y", "dx", "w_num", "w_den", "d_num", "d_den"):
        out[key] = torch.from_numpy(arr[f"{name}/{key}"].copy())
    out["dims"] = dims_of(meta["shape"], meta["layout"])
    return out


def load_cfg1() -> dict:
    return dict(np.load(os.path.join(GOLDEN_DIR, "golden_cfg1.npz")))


def dims_of(shape, layout: str):
    shape = list(shape)
    if layout == "nchw":
        return shape[0], shape[1], shape[2] * shape[3]
    c = shape[-1]
    n = int(np.prod(shape))
    return n // c, c, 1
