"""Host-side launchers and autograd Functions over the C ABI.

Mirrors the reference's launcher/Function layer for the group-rational path:

  rational_fwd_cuda / rational_bwd_cuda        <- kat_rational/rational_triton.py:76-94, 217-238
  rational_fwd_cuda_2d / rational_bwd_cuda_2d  <- kat_rational/rational_triton2d.py:71-91, 194-220
  RationalCUDA1DGroup (alias RationalTriton1DGroup) <- kat_rational/rational_triton.py:241-297
  RationalCUDA2D (alias RationalTriton2D)      <- kat_rational/rational_triton2d.py:226-246

Same argument meaning: `n` is the [group, 6] numerator (the module passes its
[1, 6] parameter repeated per group), `d` the [group, 4] denominator; the
backward returns (d_x, d_n[group, 6] fp32, d_d[group, 4] fp32).  The math is the
reference's PyTorch formula (kat_rational/kat_1dgroup_torch.py:27-78), computed
by the sm_100a kernels in libkat_rational.so; nothing here computes on the CPU.
"""

from __future__ import annotations

import ctypes
import os

import torch
from torch import Tensor

from . import _native

# KAT_RATIONAL_NVTX=1: every forward / backward call of the library is wrapped in an NVTX range
# ("kat_rational.fwd [shape] dtype" / "kat_rational.bwd ..."), so profiler timelines and ncu
# --nvtx filters can attribute kernels to module calls.  Off by default (no per-call cost).
_NVTX = os.environ.get("KAT_RATIONAL_NVTX", "") == "1"


def _nvtx_push(kind: str, x: Tensor) -> None:
    torch.cuda.nvtx.range_push(f"kat_rational.{kind} {list(x.shape)} {str(x.dtype)[6:]}")

_DTYPE_CODES = {
    torch.float32: _native.KAT_DTYPE_F32,
    torch.float16: _native.KAT_DTYPE_F16,
    torch.bfloat16: _native.KAT_DTYPE_BF16,
}

_workspace_cache: dict = {}


def _dtype_code(t: Tensor) -> int:
    try:
        return _DTYPE_CODES[t.dtype]
    except KeyError:
        raise TypeError(f"kat_rational: unsupported dtype {t.dtype} "
                        f"(expected float32, float16 or bfloat16)") from None


def _check_cuda(name: str, t: Tensor) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"kat_rational: {name} must be a CUDA tensor (got device {t.device}); "
                           f"the CUDA path has no CPU implementation")


def _shared(formula: int) -> bool:
    return bool(formula & _native.KAT_SHARED_NUMERATOR)


def _check_counts(n: Tensor, d: Tensor, group: int, shared: bool = False) -> None:
    n_rows = 1 if shared else group
    assert n.numel() == n_rows * 6, f"numerator: expected {n_rows*6} coeffs, got {n.numel()}"
    assert d.numel() == group * 4, f"denominator: expected {group*4} coeffs, got {d.numel()}"


def _coefficients(n: Tensor, d: Tensor, group: int, device: torch.device, shared: bool = False):
    _check_counts(n, d, group, shared)
    n32 = n.detach().to(device=device, dtype=torch.float32).contiguous()
    d32 = d.detach().to(device=device, dtype=torch.float32).contiguous()
    return n32, d32


def _dims_1d(x: Tensor, group: int):
    if x.dim() < 1:
        raise ValueError("kat_rational: input must have a channel dimension")
    channels = x.shape[-1]
    if group < 1 or channels % group != 0:
        raise ValueError(f"kat_rational: channels ({channels}) must be divisible by "
                         f"num_groups ({group})")
    batch = x.numel() // channels if channels else 0
    return batch, channels, 1


def _dims_2d(x: Tensor, group: int):
    if x.dim() != 4:
        raise ValueError(f"kat_rational: 2D input must be [B, C, H, W], got {tuple(x.shape)}")
    b, c, h, w = x.shape
    if group < 1 or c % group != 0:
        raise ValueError(f"kat_rational: channels ({c}) must be divisible by num_groups ({group})")
    return b, c, h * w


def _stream_ptr(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _workspace_bytes(dims, group: int, code: int, device: torch.device) -> int:
    key = (dims, group, code, device.index)
    hit = _workspace_cache.get(key)
    if hit is not None:
        return hit
    out = ctypes.c_size_t(0)
    _native.check("kat_rational_bwd_workspace_size",
                  _native.lib().kat_rational_bwd_workspace_size(
                      dims[0], dims[1], dims[2], group, code, device.index, ctypes.byref(out)))
    _workspace_cache[key] = out.value
    return out.value


def _fwd_f64(x: Tensor, n: Tensor, d: Tensor, group: int, dims, formula: int) -> Tensor:
    """float64 tensors: the float64 forward kernel (kat_rational_fwd_f64)."""
    x = x.contiguous()
    n64 = n.detach().to(device=x.device, dtype=torch.float64).contiguous()
    d64 = d.detach().to(device=x.device, dtype=torch.float64).contiguous()
    y = torch.empty_like(x, memory_format=torch.contiguous_format)
    with torch.cuda.device(x.device):
        status = _native.lib().kat_rational_fwd_f64(
            x.data_ptr(), y.data_ptr(), n64.data_ptr(), d64.data_ptr(), dims[0], dims[1],
            dims[2], group, formula, _stream_ptr(x.device))
    _native.check("kat_rational_fwd_f64", status)
    return y


def _fwd(x: Tensor, n: Tensor, d: Tensor, group: int, dims,
         formula: int = _native.KAT_FORMULA_KAT) -> Tensor:
    shared = _shared(formula)
    _check_counts(n, d, group, shared)
    _check_cuda("input", x)
    if x.dtype == torch.float64:
        if shared:
            n, formula = n.reshape(1, 6).expand(group, 6), formula & ~_native.KAT_SHARED_NUMERATOR
        return _fwd_f64(x, n, d, group, dims, formula)
    code = _dtype_code(x)
    x = x.contiguous()
    n32, d32 = _coefficients(n, d, group, x.device, shared)
    y = torch.empty_like(x, memory_format=torch.contiguous_format)
    if _NVTX:
        _nvtx_push("fwd", x)
    with torch.cuda.device(x.device):
        args = (x.data_ptr(), y.data_ptr(), n32.data_ptr(), d32.data_ptr(),
                dims[0], dims[1], dims[2], group, code)
        if formula == _native.KAT_FORMULA_KAT:
            status = _native.lib().kat_rational_fwd(*args, _stream_ptr(x.device))
        else:
            status = _native.lib().kat_rational_fwd_formula(*args, formula,
                                                            _stream_ptr(x.device))
    if _NVTX:
        torch.cuda.nvtx.range_pop()
    _native.check("kat_rational_fwd", status)
    return y


def _bwd(grad_output: Tensor, x: Tensor, n: Tensor, d: Tensor, group: int, dims,
         need_dx: bool = True, exchange=None, formula: int = _native.KAT_FORMULA_KAT):
    shared = _shared(formula)
    _check_counts(n, d, group, shared)
    _check_cuda("input", x)
    _check_cuda("grad_output", grad_output)
    if x.dtype == torch.float64:
        # float64 inputs: the fp32 backward (the reference's backward kernels compute in
        # fp32 too), results returned in float64.
        d_x, d_n, d_d = _bwd(grad_output.float(), x.float(), n, d, group, dims, need_dx,
                             exchange, formula)
        return (d_x.double() if d_x is not None else None), d_n, d_d
    code = _dtype_code(x)
    x = x.contiguous()
    if grad_output.dtype != x.dtype:
        grad_output = grad_output.to(x.dtype)
    grad_output = grad_output.contiguous()
    if grad_output.shape != x.shape:
        raise ValueError(f"kat_rational: grad_output shape {tuple(grad_output.shape)} != "
                         f"input shape {tuple(x.shape)}")
    n32, d32 = _coefficients(n, d, group, x.device, shared)
    d_x = torch.empty_like(x, memory_format=torch.contiguous_format) if need_dx else None
    d_n = torch.empty(n.shape, dtype=torch.float32, device=x.device)
    d_d = torch.empty(d.shape, dtype=torch.float32, device=x.device)
    if exchange is not None and (formula & ~_native.KAT_SHARED_NUMERATOR) != _native.KAT_FORMULA_KAT:
        raise ValueError("kat_rational: the fused exchange computes the KAT formula only")
    if _NVTX:
        _nvtx_push("bwd", x)
    with torch.cuda.device(x.device):
        ws_bytes = _workspace_bytes(dims, group, code, x.device)
        ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=x.device)
        args = (x.data_ptr(), grad_output.data_ptr(),
                d_x.data_ptr() if d_x is not None else None, n32.data_ptr(), d32.data_ptr(),
                d_n.data_ptr(), d_d.data_ptr(), ws.data_ptr(), ws.numel(), dims[0], dims[1],
                dims[2], group, code)
        if exchange is None and formula != _native.KAT_FORMULA_KAT:
            status = _native.lib().kat_rational_bwd_formula(*args, formula,
                                                            _stream_ptr(x.device))
        elif exchange is None:
            status = _native.lib().kat_rational_bwd(*args, _stream_ptr(x.device))
        elif formula == _native.KAT_FORMULA_KAT:
            status = _native.lib().kat_rational_bwd_allreduce(
                *args, ctypes.byref(exchange.peers), _stream_ptr(x.device))
        else:
            status = _native.lib().kat_rational_bwd_allreduce_formula(
                *args, formula, ctypes.byref(exchange.peers), _stream_ptr(x.device))
    if _NVTX:
        torch.cuda.nvtx.range_pop()
    _native.check("kat_rational_bwd", status)
    return d_x, d_n, d_d


def rational_fwd_cuda(x: Tensor, n: Tensor, d: Tensor, group: int) -> Tensor:
    """Forward for channels-last input ([..., C]); kat_rational/rational_triton.py:76-94."""
    return _fwd(x, n, d, group, _dims_1d(x, group))


def rational_bwd_cuda(grad_output: Tensor, x: Tensor, n: Tensor, d: Tensor, group: int):
    """Backward for channels-last input; kat_rational/rational_triton.py:217-238.

    Returns (d_x, d_n, d_d) with d_n/d_d fp32 and shaped like n/d.
    """
    return _bwd(grad_output, x, n, d, group, _dims_1d(x, group))


def rational_fwd_cuda_2d(x: Tensor, n: Tensor, d: Tensor, group: int) -> Tensor:
    """Forward for NCHW input; kat_rational/rational_triton2d.py:71-91."""
    return _fwd(x, n, d, group, _dims_2d(x, group))


def rational_bwd_cuda_2d(grad_output: Tensor, x: Tensor, n: Tensor, d: Tensor, group: int):
    """Backward for NCHW input; kat_rational/rational_triton2d.py:194-220."""
    return _bwd(grad_output, x, n, d, group, _dims_2d(x, group))


class RationalCUDA1DGroup(torch.autograd.Function):
    """Group-rational activation on channels-last input ([B, L, C] or [B, C]).

    Drop-in for the reference's RationalTriton1DGroup (kat_rational/rational_triton.py:241-297):
    same apply(input, weight_numerator[G,6], weight_denominator[G,4], group) signature, the
    same custom_fwd(cast_inputs=float32) / custom_bwd autocast behaviour, and the backward
    returns (d_input, d_numerator[G,6], d_denominator[G,4], None).
    """

    @staticmethod
    @torch.amp.custom_fwd(cast_inputs=torch.float32, device_type="cuda")
    def forward(ctx, input: Tensor, weight_numerator: Tensor, weight_denominator: Tensor,
                group: int) -> Tensor:
        ctx.save_for_backward(input, weight_numerator, weight_denominator)
        ctx.group = group
        return rational_fwd_cuda(input, weight_numerator, weight_denominator, group)

    @staticmethod
    @torch.amp.custom_bwd(device_type="cuda")
    def backward(ctx, grad_output: Tensor):
        input, weight_numerator, weight_denominator = ctx.saved_tensors
        group = ctx.group
        d_input, d_num, d_den = _bwd(grad_output, input, weight_numerator, weight_denominator,
                                     group, _dims_1d(input, group),
                                     need_dx=ctx.needs_input_grad[0])
        return d_input, d_num, d_den, None


class RationalCUDA2D(torch.autograd.Function):
    """Group-rational activation on NCHW input ([B, C, H, W]).

    Drop-in for the reference's RationalTriton2D (kat_rational/rational_triton2d.py:226-246).
    """

    @staticmethod
    @torch.amp.custom_fwd(cast_inputs=torch.float32, device_type="cuda")
    def forward(ctx, input: Tensor, weight_numerator: Tensor, weight_denominator: Tensor,
                group: int) -> Tensor:
        ctx.save_for_backward(input, weight_numerator, weight_denominator)
        ctx.group = group
        return rational_fwd_cuda_2d(input, weight_numerator, weight_denominator, group)

    @staticmethod
    @torch.amp.custom_bwd(device_type="cuda")
    def backward(ctx, grad_output: Tensor):
        input, weight_numerator, weight_denominator = ctx.saved_tensors
        group = ctx.group
        d_input, d_num, d_den = _bwd(grad_output, input, weight_numerator, weight_denominator,
                                     group, _dims_2d(input, group),
                                     need_dx=ctx.needs_input_grad[0])
        return d_input, d_num, d_den, None


_KAT_SHARED = _native.KAT_FORMULA_KAT | _native.KAT_SHARED_NUMERATOR

# The shared-row grid reduction runs in one block of 8 warps, each summing its groups one after
# the other: up to 16 groups (two per warp) it costs no more than the per-group reduction; above
# that the modules repeat the numerator per group and let torch sum its gradient instead.
SHARED_ROW_MAX_GROUPS = 16


class KatGroupFunction(torch.autograd.Function):
    """The Function KAT_Group / KAT_Group2D apply on the CUDA kernels: the module's
    weight_numerator [1, 6] reaches the kernels as one row shared by every group
    (KAT_SHARED_NUMERATOR), so the reference's per-forward repeat to [G, 6]
    (kat_rational/kat_1dgroup_triton.py:86) and its backward (a sum over groups) do not run as
    separate launches: the grid reduction writes d_numerator [1, 6] summed over groups in a
    fixed fp64 order.  Values and d_input, d_denominator equal RationalCUDA1DGroup /
    RationalCUDA2D on the repeated numerator bit for bit.  `nchw` selects the [B, C, H, W]
    layout; with `exchange` (a distributed.PeerExchange) the backward also exchanges the
    coefficient gradients with the other ranks (kat_rational_bwd_allreduce_formula), summing the
    numerator over groups in the same order as the local backward.  shared=False takes the
    reference's contract instead (numerator [G, 6], d_numerator [G, 6])."""

    @staticmethod
    @torch.amp.custom_fwd(cast_inputs=torch.float32, device_type="cuda")
    def forward(ctx, input: Tensor, weight_numerator: Tensor, weight_denominator: Tensor,
                group: int, nchw: bool = False, exchange=None, shared: bool = True) -> Tensor:
        ctx.save_for_backward(input, weight_numerator, weight_denominator)
        ctx.group = group
        ctx.nchw = nchw
        ctx.exchange = exchange
        ctx.formula = _KAT_SHARED if shared else _native.KAT_FORMULA_KAT
        dims = _dims_2d(input, group) if nchw else _dims_1d(input, group)
        return _fwd(input, weight_numerator, weight_denominator, group, dims, ctx.formula)

    @staticmethod
    @torch.amp.custom_bwd(device_type="cuda")
    def backward(ctx, grad_output: Tensor):
        input, weight_numerator, weight_denominator = ctx.saved_tensors
        group = ctx.group
        dims = _dims_2d(input, group) if ctx.nchw else _dims_1d(input, group)
        d_input, d_num, d_den = _bwd(grad_output, input, weight_numerator, weight_denominator,
                                     group, dims, need_dx=ctx.needs_input_grad[0],
                                     exchange=ctx.exchange, formula=ctx.formula)
        return d_input, d_num, d_den, None, None, None, None


# The reference's export names (kat_rational/__init__.py:2, rational_triton2d.py:226).
RationalTriton1DGroup = RationalCUDA1DGroup
RationalTriton2D = RationalCUDA2D
