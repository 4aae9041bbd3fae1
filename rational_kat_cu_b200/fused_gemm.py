"""GEMMs with the group-rational activation fused into the epilogue, and the GR-KAN MLP block
(fc1 -> act2 -> fc2) built on them.

The reference's KAN block (README.md:20-51) is act1 -> drop -> fc1 -> act2 -> drop -> fc2 with
act2 a `KAT_Group` (kat_rational/kat_1dgroup_triton.py:46-87).  act2 sits between two GEMMs,
so here its forward runs in fc1's epilogue and its backward in the epilogue of fc2's
input-gradient GEMM (sm_100a tcgen05 kernels of libkat_rational.so, include/kat_gemm.h):

  forward   h, y = kat_gemm_rational_fwd(x, W1, b1)     h = x W1^T + b1, y = act2(h)
            out  = y W2^T + b2                           (cuBLAS)
  backward  dW2 = g^T y, db2 = sum g                     (cuBLAS / torch)
            dh, d_num, d_den = kat_gemm_rational_bwd(g, W2^T, h)
            dW1 = dh^T x, db1 = sum dh, dx = dh W1      (cuBLAS / torch)

so the [rows, hidden] activation is written once (h, y) instead of being written by fc1 and
re-read by act2, and act2's input gradient is never stored.  All operands are bf16; the
activation coefficients are fp32 as in `KAT_Group`.  There is no CPU implementation: CPU
tensors raise, and a missing library raises on first use.
"""

from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch
import torch.nn.functional as F
from torch import Tensor

from . import _native

TILE_N = 256   # N must be a multiple of this
TILE_K = 64    # K must be a multiple of this
CHUNK = 32     # N / num_groups must be a multiple of this


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _mat(t: Tensor, name: str) -> Tensor:
    if not t.is_cuda:
        raise RuntimeError(f"fused_gemm: {name} must be a CUDA tensor; there is no CPU "
                           f"implementation")
    if t.dtype != torch.bfloat16:
        raise TypeError(f"fused_gemm: {name} must be bfloat16, got {t.dtype}")
    if t.dim() != 2:
        raise ValueError(f"fused_gemm: {name} must be 2-D, got shape {tuple(t.shape)}")
    return t.contiguous()


def _shapes(a: Tensor, b: Tensor) -> Tuple[int, int, int]:
    m, k = a.shape
    n, k2 = b.shape
    if k != k2:
        raise ValueError(f"fused_gemm: inner dimensions differ: a {tuple(a.shape)}, "
                         f"b {tuple(b.shape)}")
    if n % TILE_N or k % TILE_K or m < 0:
        raise ValueError(f"fused_gemm: need N % {TILE_N} == 0 and K % {TILE_K} == 0, got "
                         f"M={m}, N={n}, K={k}")
    return m, n, k


def supports(m: int, n: int, k: int, num_groups: int = 1) -> bool:
    """Whether the fused kernels take an [m, k] x [n, k]^T problem with num_groups groups."""
    return (m >= 0 and n % TILE_N == 0 and k % TILE_K == 0 and num_groups >= 1
            and n % num_groups == 0 and (n // num_groups) % CHUNK == 0)


def _coef(num: Tensor, den: Tensor, num_groups: int, n: int):
    nf = num.detach().float().contiguous()
    df = den.detach().float().contiguous()
    if tuple(nf.shape) != (num_groups, 6) or tuple(df.shape) != (num_groups, 4):
        raise ValueError(f"fused_gemm: expected numerator [{num_groups}, 6] and denominator "
                         f"[{num_groups}, 4], got {tuple(nf.shape)} and {tuple(df.shape)}")
    if not nf.is_cuda or not df.is_cuda:
        raise RuntimeError("fused_gemm: coefficients must be CUDA tensors")
    if n % num_groups or (n // num_groups) % CHUNK:
        raise ValueError(f"fused_gemm: N={n} must split into {num_groups} groups of a multiple "
                         f"of {CHUNK} columns")
    return nf, df


def gemm_bf16(a: Tensor, b: Tensor, bias: Optional[Tensor] = None) -> Tensor:
    """C = a b^T (+ bias), a [M, K], b [N, K], bf16 in and out, fp32 accumulation."""
    a = _mat(a, "a")
    b = _mat(b, "b")
    m, n, k = _shapes(a, b)
    if bias is not None:
        bias = bias.detach().to(torch.bfloat16).contiguous()
    c = torch.empty(m, n, device=a.device, dtype=torch.bfloat16)
    if m == 0:
        return c
    with torch.cuda.device(a.device):
        st = _native.lib().kat_gemm_bf16(a.data_ptr(), b.data_ptr(),
                                         bias.data_ptr() if bias is not None else None,
                                         c.data_ptr(), m, n, k, _stream(a.device))
    _native.check("kat_gemm_bf16", st)
    return c


def gemm_rational_fwd(a: Tensor, b: Tensor, bias: Optional[Tensor], num: Tensor, den: Tensor,
                      num_groups: int, formula: int = _native.KAT_FORMULA_KAT,
                      need_h: bool = True) -> Tuple[Optional[Tensor], Tensor]:
    """h = a b^T + bias and y = P(h)/Q(h) per column group; returns (h, y), both bf16 [M, N].
    With need_h=False (no backward follows) only y is written and h is None."""
    a = _mat(a.detach(), "a")
    b = _mat(b.detach(), "b")
    m, n, k = _shapes(a, b)
    nf, df = _coef(num, den, num_groups, n)
    if bias is not None:
        bias = bias.detach().to(torch.bfloat16).contiguous()
    y = torch.empty(m, n, device=a.device, dtype=torch.bfloat16)
    h = torch.empty_like(y) if need_h else None
    if m == 0:
        return h, y
    with torch.cuda.device(a.device):
        st = _native.lib().kat_gemm_rational_fwd(
            a.data_ptr(), b.data_ptr(), bias.data_ptr() if bias is not None else None,
            nf.data_ptr(), df.data_ptr(), h.data_ptr() if h is not None else None,
            y.data_ptr(), m, n, k, num_groups, formula, _stream(a.device))
    _native.check("kat_gemm_rational_fwd", st)
    return h, y


def gemm_rational_bwd(a: Tensor, b: Tensor, h: Tensor, num: Tensor, den: Tensor,
                      num_groups: int, formula: int = _native.KAT_FORMULA_KAT
                      ) -> Tuple[Tensor, Tensor, Tensor]:
    """g = a b^T (not stored), dh = g * y'(h); returns (dh bf16 [M, N], d_num [G, 6] fp32,
    d_den [G, 4] fp32)."""
    a = _mat(a.detach(), "a")
    b = _mat(b.detach(), "b")
    h = _mat(h.detach(), "h")
    m, n, k = _shapes(a, b)
    if tuple(h.shape) != (m, n):
        raise ValueError(f"fused_gemm: h shape {tuple(h.shape)} != {(m, n)}")
    nf, df = _coef(num, den, num_groups, n)
    dev = a.device
    if m == 0:  # sums over no elements
        return (torch.empty(0, n, device=dev, dtype=torch.bfloat16),
                torch.zeros(num_groups, 6, device=dev), torch.zeros(num_groups, 4, device=dev))
    lib = _native.lib()
    ws_bytes = lib.kat_gemm_rational_bwd_workspace_bytes(m, n, num_groups, dev.index or 0)
    if ws_bytes == 0:
        raise RuntimeError("kat_gemm_rational_bwd_workspace_bytes returned 0")
    ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8)
    dh = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
    d_num = torch.empty(num_groups, 6, device=dev, dtype=torch.float32)
    d_den = torch.empty(num_groups, 4, device=dev, dtype=torch.float32)
    with torch.cuda.device(dev):
        st = lib.kat_gemm_rational_bwd(
            a.data_ptr(), b.data_ptr(), h.data_ptr(), nf.data_ptr(), df.data_ptr(),
            dh.data_ptr(), d_num.data_ptr(), d_den.data_ptr(), ws.data_ptr(), ws_bytes,
            m, n, k, num_groups, formula, _stream(dev))
    _native.check("kat_gemm_rational_bwd", st)
    return dh, d_num, d_den


def device_status(device: int = 0, reset: bool = False) -> int:
    """Sticky status word of the GEMM kernels (0 = no pipeline wait ran out)."""
    out = ctypes.c_int(0)
    _native.check("kat_gemm_device_status",
                  _native.lib().kat_gemm_device_status(device, 1 if reset else 0,
                                                       ctypes.byref(out)))
    return out.value


class KANMlpFused(torch.autograd.Function):
    """fc1 -> act2 -> fc2 of the KAN block with act2 in the GEMM epilogues.

    Inputs: x [M, C] bf16, fc1 weight [H, C] / bias [H], act2 numerator repeated per group
    [G, 6] and denominator [G, 4] (as `KAT_Group.forward` passes them,
    kat_1dgroup_triton.py:86-87), fc2 weight [C, H] / bias [C]."""

    @staticmethod
    def forward(ctx, x: Tensor, w1: Tensor, b1: Optional[Tensor], num: Tensor, den: Tensor,
                w2: Tensor, b2: Optional[Tensor], num_groups: int,
                formula: int = _native.KAT_FORMULA_KAT) -> Tensor:
        h, y = gemm_rational_fwd(x, w1, b1, num, den, num_groups, formula)
        out = F.linear(y, w2, b2)
        ctx.save_for_backward(x, w1, h, y, w2, num, den)
        ctx.num_groups = num_groups
        ctx.formula = formula
        ctx.has_b1 = b1 is not None
        ctx.has_b2 = b2 is not None
        return out

    @staticmethod
    def backward(ctx, g_out: Tensor):
        x, w1, h, y, w2, num, den = ctx.saved_tensors
        g = g_out.contiguous()
        d_w2 = g.t() @ y
        d_b2 = g.sum(0) if ctx.has_b2 else None
        dh, d_num, d_den = gemm_rational_bwd(g, w2.t().contiguous(), h, num, den,
                                             ctx.num_groups, ctx.formula)
        d_w1 = dh.t() @ x
        d_b1 = dh.sum(0) if ctx.has_b1 else None
        dx = dh @ w1
        return (dx, d_w1, d_b1, d_num.to(num.dtype), d_den.to(den.dtype), d_w2, d_b2, None,
                None)


def kan_mlp_fused(x: Tensor, fc1: torch.nn.Linear, act2, fc2: torch.nn.Linear) -> Tensor:
    """fc2(act2(fc1(x))) for x [..., C] through `KANMlpFused` (act2 a `KAT_Group`).  When no
    gradient is needed (inference) the forward GEMM writes y only."""
    shape = x.shape
    x2 = x.reshape(-1, shape[-1])
    g = act2.num_groups
    params = (x, fc1.weight, fc1.bias, act2.weight_numerator, act2.weight_denominator,
              fc2.weight, fc2.bias)
    if not (torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in params)):
        _, y = gemm_rational_fwd(x2, fc1.weight, fc1.bias, act2.weight_numerator.repeat(g, 1),
                                 act2.weight_denominator, g, need_h=False)
        out = F.linear(y, fc2.weight, fc2.bias)
        return out.reshape(*shape[:-1], out.shape[-1])
    out = KANMlpFused.apply(x2, fc1.weight, fc1.bias, act2.weight_numerator.repeat(g, 1),
                            act2.weight_denominator, fc2.weight, fc2.bias, g,
                            _native.KAT_FORMULA_KAT)
    return out.reshape(*shape[:-1], out.shape[-1])
