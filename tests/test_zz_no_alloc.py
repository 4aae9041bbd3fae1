"""kat_rational_bwd_noalloc: the backward for callers that cannot allocate device memory
where they run it (plugin hosts whose operator interface gives the operator buffers but no
allocator, fixed-budget real-time loops where a mid-run cudaMalloc may stall or fail).  It
must give exactly the results of kat_rational_bwd with a fresh caller-allocated workspace,
on two calls in a row, also right after a call on other data, another shape and more groups
has left its partial sums in the shared scratch array; and it must reject problems whose
scratch need exceeds its fixed 2 MiB with KAT_ERR_SCRATCH_LIMIT.

Collected last (file name) so that a run stopping at the first failure has run every other
test; it also passes alone in a fresh process.
"""

import ctypes

import pytest
import torch

from rational_kat_cu_b200 import _native

pytestmark = pytest.mark.gpu

DT = {"f32": (torch.float32, _native.KAT_DTYPE_F32),
      "bf16": (torch.bfloat16, _native.KAT_DTYPE_BF16),
      "f16": (torch.float16, _native.KAT_DTYPE_F16)}

CASES = [
    # (batch, channels, inner), groups, dtype
    ((16 * 197, 3072, 1), 8, "bf16"),     # 16-byte vectors: cp.async-ring backward
    ((8 * 197, 768, 1), 8, "f32"),
    ((4, 64, 196), 8, "f32"),             # NCHW
    ((15, 36, 1), 12, "f16"),             # 3-wide groups: scalar register backward
    ((6, 768, 1), 64, "bf16"),            # 12-wide groups: 4-element vectors
]


def _inputs(dims, groups, dtype, device):
    tdt, _ = DT[dtype]
    g = torch.Generator(device="cpu").manual_seed(123)
    shape = (dims[0], dims[1] * dims[2])
    x = (torch.randn(shape, generator=g) * 1.5).to(tdt).to(device)
    gy = torch.randn(shape, generator=g).to(tdt).to(device)
    num = (torch.randn(groups, 6, generator=g) * 0.3).to(device)
    den = (torch.randn(groups, 4, generator=g) * 0.3).to(device)
    return x, gy, num, den


def _outputs(x, groups, device):
    return (torch.empty_like(x), torch.empty(groups, 6, device=device),
            torch.empty(groups, 4, device=device))


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def bwd_with_workspace(x, gy, num, den, dims, groups, code, device):
    """kat_rational_bwd with a fresh workspace whose bytes are all 0xFF (NaN doubles), so a
    read of any slot the call did not write would show in its results."""
    lib = _native.lib()
    need = ctypes.c_size_t(0)
    _native.check("workspace", lib.kat_rational_bwd_workspace_size(
        dims[0], dims[1], dims[2], groups, code, device.index or 0, ctypes.byref(need)))
    ws = torch.full((max(need.value, 16),), 0xFF, dtype=torch.uint8, device=device)
    dx, dn, dd = _outputs(x, groups, device)
    _native.check("kat_rational_bwd", lib.kat_rational_bwd(
        x.data_ptr(), gy.data_ptr(), dx.data_ptr(), num.data_ptr(), den.data_ptr(),
        dn.data_ptr(), dd.data_ptr(), ws.data_ptr(), ws.numel(), dims[0], dims[1], dims[2],
        groups, code, _stream()))
    torch.cuda.synchronize()
    return dx, dn, dd


def bwd_noalloc(x, gy, num, den, dims, groups, code, device):
    dx, dn, dd = _outputs(x, groups, device)
    status = _native.lib().kat_rational_bwd_noalloc(
        x.data_ptr(), gy.data_ptr(), dx.data_ptr(), num.data_ptr(), den.data_ptr(),
        dn.data_ptr(), dd.data_ptr(), dims[0], dims[1], dims[2], groups, code, _stream())
    _native.check("kat_rational_bwd_noalloc", status)
    torch.cuda.synchronize()
    return dx, dn, dd


# A call on other data, with more groups and another shape, that fills far more scratch
# slots (blocks x segments x local groups: about 1.5 MiB of the 2 MiB) than any case below
# reads (at most about 0.5 MiB).
POLLUTER = ((96, 3072, 1), 96, "f32")


def _pollute(device):
    dims, groups, dtype = POLLUTER
    _, code = DT[dtype]
    x, gy, num, den = _inputs(dims, groups, dtype, device)
    x.mul_(3.0).add_(0.5)
    out = bwd_noalloc(x, gy, num, den, dims, groups, code, device)
    assert torch.isfinite(out[1]).all()


def _assert_identical(got, want, label):
    for g, w, name in zip(got, want, ("dx", "d_num", "d_den")):
        assert torch.equal(g, w), f"{label}: {name} differs from the workspace entry point"


@pytest.mark.parametrize("dims,groups,dtype", CASES)
def test_noalloc_matches_workspace_entry_point(dims, groups, dtype):
    device = torch.device("cuda", 0)
    _, code = DT[dtype]
    x, gy, num, den = _inputs(dims, groups, dtype, device)
    ref = bwd_with_workspace(x, gy, num, den, dims, groups, code, device)
    _pollute(device)
    for call in range(2):
        out = bwd_noalloc(x, gy, num, den, dims, groups, code, device)
        _assert_identical(out, ref, f"call {call} after a larger call")
    assert _native.device_status(0) == 0


def test_noalloc_rejects_problems_beyond_its_scratch():
    """One group per channel over 4096 channels needs far more than 2 MiB of partial sums."""
    device = torch.device("cuda", 0)
    dims, groups = (64, 4096, 1), 4096
    lib = _native.lib()
    need = ctypes.c_size_t(0)
    _native.check("workspace", lib.kat_rational_bwd_workspace_size(
        dims[0], dims[1], dims[2], groups, _native.KAT_DTYPE_F32, 0, ctypes.byref(need)))
    assert need.value > (2 << 20)
    x, gy, num, den = _inputs(dims, groups, "f32", device)
    dx, dn, dd = _outputs(x, groups, device)
    status = lib.kat_rational_bwd_noalloc(
        x.data_ptr(), gy.data_ptr(), dx.data_ptr(), num.data_ptr(), den.data_ptr(),
        dn.data_ptr(), dd.data_ptr(), dims[0], dims[1], dims[2], groups, _native.KAT_DTYPE_F32,
        _stream())
    assert status == _native.KAT_ERR_SCRATCH_LIMIT
    assert "2 MiB" in _native.strerror(status)
