"""ORACLE — test infrastructure only (tests/, __graft_entry__.smoke(), bench.py CPU leg).

ctypes wrapper of the float64 restatement in kat_oracle.c (formula of the reference's
kat_rational/kat_1dgroup_torch.py:27-78 and its autograd gradients).  Inputs are the
fp32 values the kernels consume (16-bit inputs upcast exactly); outputs are float64
numpy arrays plus the magnitude sums used by the condition-aware tolerances.
"""

from __future__ import annotations

import ctypes

import numpy as np

from . import build as _build

_lib = None


def lib():
    global _lib
    if _lib is None:
        handle = ctypes.CDLL(_build.build())
        vp, i64 = ctypes.c_void_p, ctypes.c_int64
        handle.kat_oracle_forward.argtypes = [vp, i64, i64, i64, i64, vp, vp, vp, vp]
        handle.kat_oracle_forward.restype = None
        handle.kat_oracle_backward.argtypes = [vp, vp, i64, i64, i64, i64, vp, vp,
                                               vp, vp, vp, vp, vp, vp]
        handle.kat_oracle_backward.restype = None
        handle.kat_oracle_threads.restype = ctypes.c_int
        _lib = handle
    return _lib


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def forward(x, w_num, w_den, dims, groups):
    """x: flat fp32 values of a contiguous [batch, channels, inner] tensor.
    w_num: [groups, 6] (or [1, 6], repeated), w_den: [groups, 4].
    Returns (y, y_mag) float64 arrays shaped like x."""
    x = _f32(x)
    wn = _f32(np.broadcast_to(np.asarray(w_num, np.float32).reshape(-1, 6), (groups, 6)))
    wd = _f32(np.asarray(w_den, np.float32).reshape(groups, 4))
    y = np.empty(x.shape, np.float64)
    ym = np.empty(x.shape, np.float64)
    lib().kat_oracle_forward(_ptr(x), dims[0], dims[1], dims[2], groups, _ptr(wn), _ptr(wd),
                             _ptr(y), _ptr(ym))
    return y, ym


def backward(x, grad_out, w_num, w_den, dims, groups, want_dx: bool = True):
    """Returns dict with dx, dx_mag (None unless want_dx), d_num [G,6], d_den [G,4],
    d_num_mag, d_den_mag (float64)."""
    x = _f32(x)
    go = _f32(grad_out)
    wn = _f32(np.broadcast_to(np.asarray(w_num, np.float32).reshape(-1, 6), (groups, 6)))
    wd = _f32(np.asarray(w_den, np.float32).reshape(groups, 4))
    dx = np.empty(x.shape, np.float64) if want_dx else None
    dxm = np.empty(x.shape, np.float64) if want_dx else None
    dn = np.empty((groups, 6), np.float64)
    dd = np.empty((groups, 4), np.float64)
    dnm = np.empty((groups, 6), np.float64)
    ddm = np.empty((groups, 4), np.float64)
    lib().kat_oracle_backward(_ptr(x), _ptr(go), dims[0], dims[1], dims[2], groups, _ptr(wn),
                              _ptr(wd), _ptr(dx), _ptr(dxm), _ptr(dn), _ptr(dd), _ptr(dnm),
                              _ptr(ddm))
    return {"dx": dx, "dx_mag": dxm, "d_num": dn, "d_den": dd, "d_num_mag": dnm,
            "d_den_mag": ddm}


def threads() -> int:
    return int(lib().kat_oracle_threads())
