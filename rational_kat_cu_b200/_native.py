"""ctypes binding of libkat_rational.so (the C ABI declared in include/kat_rational.h,
include/kat_bspline.h and include/kat_gemm.h).

The library is loaded once, on first use.  If it is missing the call fails with a
RuntimeError naming the build command: there is no fallback implementation.
"""

from __future__ import annotations

import ctypes
import os
import threading

from . import _build

KAT_DTYPE_F32 = 0
KAT_DTYPE_F16 = 1
KAT_DTYPE_BF16 = 2

KAT_OK = 0
KAT_ERR_NULL_POINTER = 1
KAT_ERR_BAD_DTYPE = 2
KAT_ERR_BAD_SHAPE = 3
KAT_ERR_BAD_GROUPS = 4
KAT_ERR_WORKSPACE = 5
KAT_ERR_CUDA = 6
KAT_ERR_SCRATCH_LIMIT = 7
KAT_ERR_BAD_FORMULA = 8

KAT_FORMULA_KAT = 0
KAT_FORMULA_ABS_SUM = 1

# Every symbol include/*.h declares.
EXPORTED_SYMBOLS = (
    "kat_bspline_basis_fwd",
    "kat_bspline_basis_bwd",
    "kat_rational_fwd",
    "kat_rational_bwd",
    "kat_rational_fwd_formula",
    "kat_rational_fwd_f64",
    "kat_rational_bwd_formula",
    "kat_rational_bwd_workspace_size",
    "kat_rational_strerror",
    "kat_rational_abi_version",
    "kat_rational_make_plan",
    "kat_rational_device_status",
    "kat_rational_bwd_noalloc",
    "kat_rational_exchange_buffer_bytes",
    "kat_rational_bwd_allreduce",
    "kat_rational_exchange_grads",
    "kat_rational_bwd_allreduce_formula",
    "kat_rational_enable_peer_access",
    "kat_rational_exchange_create",
    "kat_rational_exchange_open",
    "kat_rational_exchange_close",
    "kat_rational_exchange_destroy",
    "kat_gemm_bf16",
    "kat_gemm_rational_fwd",
    "kat_gemm_rational_bwd_workspace_bytes",
    "kat_gemm_rational_bwd",
    "kat_gemm_device_status",
    "kat_gemm_set_test_stall",
)

KAT_SHARED_NUMERATOR = 0x100
KAT_MAX_PEERS = 8
KAT_DEVICE_WAIT_TIMEOUT = 1
KAT_DEVICE_EXCHANGE_TIMEOUT = 2


class KatPeers(ctypes.Structure):
    """Mirror of `kat_rational_peers`."""

    _fields_ = [
        ("world_size", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("average", ctypes.c_int32),
        ("timeout_ms", ctypes.c_int32),
        ("buffers", ctypes.c_void_p * KAT_MAX_PEERS),
    ]

ABI_VERSION = 3


class KatPlan(ctypes.Structure):
    """Mirror of `kat_rational_plan`."""

    _fields_ = [
        ("rows", ctypes.c_int64),
        ("width", ctypes.c_int64),
        ("group_width", ctypes.c_int64),
        ("num_groups", ctypes.c_int64),
        ("vec", ctypes.c_int32),
        ("threads", ctypes.c_int32),
        ("tile_cols", ctypes.c_int32),
        ("tile_rows", ctypes.c_int32),
        ("col_blocks", ctypes.c_int64),
        ("items", ctypes.c_int64),
        ("blocks", ctypes.c_int64),
        ("max_segments", ctypes.c_int32),
        ("max_local_groups", ctypes.c_int32),
        ("workspace_bytes", ctypes.c_uint64),
        ("col_block_blocks", ctypes.c_int64),
        ("col_block_extra", ctypes.c_int64),
    ]

    def as_dict(self) -> dict:
        return {name: getattr(self, name) for name, _ in self._fields_}


class KatError(RuntimeError):
    """A non-zero status returned by the C ABI."""

    def __init__(self, func: str, status: int, message: str):
        super().__init__(f"{func} failed with status {status}: {message}")
        self.status = status


_lock = threading.Lock()
_lib = None


def library_path() -> str:
    """The in-tree library, or KAT_RATIONAL_LIBRARY when set (an alternative build)."""
    return os.environ.get("KAT_RATIONAL_LIBRARY") or _build.LIBRARY


def _declare(lib: ctypes.CDLL) -> None:
    vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    lib.kat_rational_fwd.argtypes = [vp, vp, vp, vp, i64, i64, i64, i64, i32, vp]
    lib.kat_rational_fwd.restype = i32
    lib.kat_rational_bwd.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, ctypes.c_size_t,
                                     i64, i64, i64, i64, i32, vp]
    lib.kat_rational_bwd.restype = i32
    lib.kat_rational_fwd_formula.argtypes = [vp, vp, vp, vp, i64, i64, i64, i64, i32, i32, vp]
    lib.kat_rational_fwd_formula.restype = i32
    lib.kat_rational_bwd_formula.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, ctypes.c_size_t,
                                             i64, i64, i64, i64, i32, i32, vp]
    lib.kat_rational_bwd_formula.restype = i32
    lib.kat_rational_fwd_f64.argtypes = [vp, vp, vp, vp, i64, i64, i64, i64, i32, vp]
    lib.kat_rational_fwd_f64.restype = i32
    lib.kat_gemm_bf16.argtypes = [vp, vp, vp, vp, i64, i64, i64, vp]
    lib.kat_gemm_bf16.restype = i32
    lib.kat_gemm_rational_fwd.argtypes = [vp, vp, vp, vp, vp, vp, vp, i64, i64, i64,
                                          ctypes.c_int32, ctypes.c_int32, vp]
    lib.kat_gemm_rational_fwd.restype = i32
    lib.kat_gemm_rational_bwd_workspace_bytes.argtypes = [i64, i64, ctypes.c_int32, i32]
    lib.kat_gemm_rational_bwd_workspace_bytes.restype = ctypes.c_size_t
    lib.kat_gemm_rational_bwd.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, vp, ctypes.c_size_t,
                                          i64, i64, i64, ctypes.c_int32, ctypes.c_int32, vp]
    lib.kat_gemm_rational_bwd.restype = i32
    lib.kat_gemm_device_status.argtypes = [i32, i32, ctypes.POINTER(ctypes.c_int)]
    lib.kat_gemm_device_status.restype = i32
    lib.kat_gemm_set_test_stall.argtypes = [i32]
    lib.kat_gemm_set_test_stall.restype = i32
    lib.kat_bspline_basis_fwd.argtypes = [vp, vp, vp, i64, i64, ctypes.c_int32, ctypes.c_int32,
                                          vp]
    lib.kat_bspline_basis_fwd.restype = i32
    lib.kat_bspline_basis_bwd.argtypes = [vp, vp, vp, vp, i64, i64, ctypes.c_int32,
                                          ctypes.c_int32, vp]
    lib.kat_bspline_basis_bwd.restype = i32
    lib.kat_rational_bwd_workspace_size.argtypes = [i64, i64, i64, i64, i32, i32,
                                                    ctypes.POINTER(ctypes.c_size_t)]
    lib.kat_rational_bwd_workspace_size.restype = i32
    lib.kat_rational_strerror.argtypes = [i32]
    lib.kat_rational_strerror.restype = ctypes.c_char_p
    lib.kat_rational_abi_version.argtypes = []
    lib.kat_rational_abi_version.restype = i32
    lib.kat_rational_make_plan.argtypes = [i64, i64, i64, i64, i32, i32, i32, i32,
                                           ctypes.POINTER(KatPlan)]
    lib.kat_rational_make_plan.restype = i32
    lib.kat_rational_device_status.argtypes = [i32, i32, ctypes.POINTER(ctypes.c_int)]
    lib.kat_rational_device_status.restype = i32
    lib.kat_rational_bwd_noalloc.argtypes = [vp, vp, vp, vp, vp, vp, vp, i64, i64, i64, i64,
                                             i32, vp]
    lib.kat_rational_bwd_noalloc.restype = i32
    lib.kat_rational_exchange_buffer_bytes.argtypes = [i64]
    lib.kat_rational_exchange_buffer_bytes.restype = ctypes.c_size_t
    lib.kat_rational_bwd_allreduce.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, ctypes.c_size_t,
                                               i64, i64, i64, i64, i32, ctypes.POINTER(KatPeers),
                                               vp]
    lib.kat_rational_bwd_allreduce.restype = i32
    lib.kat_rational_enable_peer_access.argtypes = [i32, i32]
    lib.kat_rational_enable_peer_access.restype = i32
    lib.kat_rational_exchange_create.argtypes = [i64, ctypes.POINTER(ctypes.c_void_p), vp]
    lib.kat_rational_exchange_create.restype = i32
    lib.kat_rational_exchange_open.argtypes = [vp, vp, ctypes.POINTER(ctypes.c_void_p)]
    lib.kat_rational_exchange_open.restype = i32
    lib.kat_rational_exchange_close.argtypes = [vp]
    lib.kat_rational_exchange_close.restype = i32
    lib.kat_rational_bwd_allreduce_formula.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp,
                                                       ctypes.c_size_t, i64, i64, i64, i64, i32,
                                                       i32, vp, vp]
    lib.kat_rational_bwd_allreduce_formula.restype = i32
    lib.kat_rational_exchange_grads.argtypes = [vp, vp, i64, vp, vp]
    lib.kat_rational_exchange_grads.restype = i32
    lib.kat_rational_exchange_destroy.argtypes = [vp]
    lib.kat_rational_exchange_destroy.restype = i32


def lib() -> ctypes.CDLL:
    """The loaded library (raises RuntimeError if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = library_path()
            if not os.path.exists(path):
                raise RuntimeError(
                    f"libkat_rational.so not found at {path}; build it with "
                    f"`python -m rational_kat_cu_b200._build` (nvcc, sm_100a)")
            handle = ctypes.CDLL(path)
            _declare(handle)
            version = handle.kat_rational_abi_version()
            if version != ABI_VERSION:
                raise RuntimeError(f"{path}: ABI version {version}, expected {ABI_VERSION}")
            _lib = handle
    return _lib


def strerror(status: int) -> str:
    return lib().kat_rational_strerror(status).decode()


def check(func: str, status: int) -> None:
    if status != KAT_OK:
        raise KatError(func, status, strerror(status))


def device_status(device: int = 0, reset: bool = False) -> int:
    """Sticky device status word (0 = no kernel gave up on a bounded wait)."""
    out = ctypes.c_int(0)
    check("kat_rational_device_status",
          lib().kat_rational_device_status(device, 1 if reset else 0, ctypes.byref(out)))
    return out.value


def make_plan(batch: int, channels: int, inner: int, num_groups: int, dtype: int,
              vec: int = 0, sm_count: int = 148, ctas_per_sm: int = 1) -> dict:
    """Launch geometry the kernels use (host arithmetic only, no GPU needed)."""
    plan = KatPlan()
    check("kat_rational_make_plan",
          lib().kat_rational_make_plan(batch, channels, inner, num_groups, dtype, vec,
                                       sm_count, ctas_per_sm, ctypes.byref(plan)))
    return plan.as_dict()
