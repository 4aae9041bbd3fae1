"""Condition-aware comparison rules shared by the parity tests.

The reference evaluates P and Q as bmm dot products of stacked powers; the kernels use
Horner's rule.  Near a zero of P (or of Q) the two fp32 evaluations legitimately differ by
a few eps32 times the magnitude sum M = sum |a_k x^k| / |Q|, which can exceed any plain
relative bound on y.  So every elementwise check is against max(|ref|, M):

  fp32 y, dx      |out - ref| <= 1e-6 * max(|ref|, M)                     (the 1e-6 relative bar)
  bf16/fp16 y,dx  |out - round(ref32)| <= 1 ulp_out(|ref|) + 1e-6 * M     (1 ulp of the output)
  coefficient     |out - ref64| <= 1e-4 * max(|ref64|, 1e-2 * S)          (1e-4 relative bar;
  gradients                                                               S = sum of |terms|)

NaN must match NaN and +-inf must match the same infinity.
"""

from __future__ import annotations

import numpy as np

FP32_RTOL = 1e-6
COEF_RTOL = 1e-4
COEF_MAG_FRAC = 1e-2


def _as64(a) -> np.ndarray:
    if hasattr(a, "detach"):
        a = a.detach().cpu().float().numpy()
    return np.asarray(a, dtype=np.float64).reshape(-1)


def check_classes(out: np.ndarray, ref: np.ndarray, name: str) -> np.ndarray:
    """Assert NaN/inf classes agree; return the mask of finite reference entries."""
    nan_o, nan_r = np.isnan(out), np.isnan(ref)
    assert np.array_equal(nan_o, nan_r), \
        f"{name}: NaN pattern differs ({nan_o.sum()} vs {nan_r.sum()})"
    inf_r = np.isinf(ref)
    if inf_r.any():
        assert np.array_equal(out[inf_r], ref[inf_r]), f"{name}: infinities differ"
    fin = np.isfinite(ref)
    assert np.isfinite(out[fin]).all(), f"{name}: non-finite output where the reference is finite"
    return fin


def ulp(values: np.ndarray, dtype: str) -> np.ndarray:
    """Spacing of the output dtype at |values| (normal range)."""
    mant = {"f32": 23, "bf16": 7, "f16": 10}[dtype]
    min_exp = {"f32": -126, "bf16": -126, "f16": -14}[dtype]
    a = np.abs(values)
    with np.errstate(divide="ignore"):
        e = np.floor(np.log2(np.where(a > 0, a, 1.0)))
    e = np.maximum(e, min_exp)
    return np.ldexp(1.0, (e - mant).astype(np.int64))


def assert_elementwise(out, ref, mag, dtype: str, name: str, ref_rounded=None) -> dict:
    """Elementwise parity of y or dx.  `ref` is the float64 (or fp32) reference value,
    `mag` its magnitude sum, `ref_rounded` the reference rounded to the output dtype."""
    o, r, m = _as64(out), _as64(ref), _as64(mag)
    fin = check_classes(o, r if ref_rounded is None else _as64(ref_rounded), name)
    fin &= np.isfinite(r) & np.isfinite(m)
    o, r, m = o[fin], r[fin], m[fin]
    scale = np.maximum(np.abs(r), m)
    if dtype == "f32":
        err = np.abs(o - r)
        tol = FP32_RTOL * scale
    else:
        rr = _as64(ref_rounded)[fin]
        err = np.abs(o - rr)
        tol = ulp(r, dtype) + FP32_RTOL * m
    bad = err > tol
    worst = float(np.max(err / np.maximum(tol, 1e-300))) if err.size else 0.0
    assert not bad.any(), (f"{name}: {int(bad.sum())}/{err.size} elements out of tolerance; "
                           f"worst err/tol = {worst:.3g}")
    return {"worst_err_over_tol": worst,
            "max_scaled_err": float(np.max(err / np.maximum(scale, 1e-300))) if err.size else 0.0}


def assert_coef_grads(out, ref64, mag, name: str) -> dict:
    o, r, m = _as64(out), _as64(ref64), _as64(mag)
    fin = check_classes(o, r, name)
    o, r, m = o[fin], r[fin], m[fin]
    tol = COEF_RTOL * np.maximum(np.abs(r), COEF_MAG_FRAC * m)
    err = np.abs(o - r)
    bad = err > tol
    assert not bad.any(), (f"{name}: coefficient gradients out of tolerance: max rel "
                           f"{float(np.max(err / np.maximum(np.abs(r), 1e-300))):.3g}, "
                           f"worst err/tol {float(np.max(err / np.maximum(tol, 1e-300))):.3g}")
    rel = err / np.maximum(np.abs(r), 1e-300)
    return {"max_rel": float(np.max(rel)) if rel.size else 0.0}
