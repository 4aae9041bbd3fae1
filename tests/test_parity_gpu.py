"""Parity of the sm_100a kernels (through the modules, the autograd Functions and the C ABI)
with the reference on the committed golden vectors, plus the edge cases.

Reference values: the reference's own fp32 outputs (golden vectors) and the float64
restatement (oracle/kat_oracle.c) for the magnitudes and the coefficient gradients.
Tolerances (tests/tolerances.py): fp32 1e-6 x max(|ref|, M); bf16/fp16 1 ulp of the output
dtype (+1e-6 M); coefficient gradients 1e-4 relative (vs float64).
"""

import ctypes

import numpy as np
import pytest
import torch

import rational_kat_cu_b200 as kat
from golden_data import TORCH_DTYPES, case_names, load_case
from oracle import c_oracle
from rational_kat_cu_b200 import _native
from tolerances import assert_coef_grads, assert_elementwise

pytestmark = pytest.mark.gpu


def _module_for(layout, groups, device):
    cls = kat.KAT_Group2D if layout == "nchw" else kat.KAT_Group
    return cls(num_groups=groups, mode="gelu").to(device)


def run_module(x, gy, w_num, w_den, groups, layout, device, dtype=torch.float32):
    mod = _module_for(layout, groups, device)
    with torch.no_grad():
        mod.weight_numerator.copy_(w_num)
        mod.weight_denominator.copy_(w_den)
    xd = x.to(device=device, dtype=dtype).requires_grad_(True)
    y = mod(xd)
    y.backward(gy.to(device=device, dtype=dtype))
    torch.cuda.synchronize()
    return y.detach(), xd.grad, mod.weight_numerator.grad, mod.weight_denominator.grad


def oracle_for(x, gy, w_num, w_den, dims, groups):
    xf = x.float().reshape(-1).cpu().numpy()
    y, ymag = c_oracle.forward(xf, w_num.cpu().numpy(), w_den.cpu().numpy(), dims, groups)
    b = c_oracle.backward(xf, gy.float().reshape(-1).cpu().numpy(), w_num.cpu().numpy(),
                          w_den.cpu().numpy(), dims, groups)
    return y, ymag, b


def assert_parity(out, ref32, oracle, dtype, name):
    """out = (y, dx, d_num[1,6], d_den[G,4]); ref32 = reference fp32 (y, dx) or None."""
    y, dx, dn, dd = out
    y64, ymag, b = oracle
    if dtype == "f32":
        assert_elementwise(y, y64, ymag, "f32", f"{name}/y vs float64")
        assert_elementwise(dx, b["dx"], b["dx_mag"], "f32", f"{name}/dx vs float64")
        if ref32 is not None:
            assert_elementwise(y, ref32[0], ymag, "f32", f"{name}/y vs reference")
            assert_elementwise(dx, ref32[1], b["dx_mag"], "f32", f"{name}/dx vs reference")
    else:
        tdt = TORCH_DTYPES[dtype]
        r_y = ref32[0] if ref32 is not None else torch.from_numpy(y64).float()
        r_dx = ref32[1] if ref32 is not None else torch.from_numpy(b["dx"]).float()
        assert_elementwise(y, r_y, ymag, dtype, f"{name}/y", ref_rounded=r_y.to(tdt).float())
        assert_elementwise(dx, r_dx, b["dx_mag"], dtype, f"{name}/dx",
                           ref_rounded=r_dx.to(tdt).float())
    assert_coef_grads(dn, b["d_num"].sum(0, keepdims=True), b["d_num_mag"].sum(0, keepdims=True),
                      f"{name}/d_num")
    assert_coef_grads(dd, b["d_den"], b["d_den_mag"], f"{name}/d_den")


def test_native_library_is_loaded(cuda_device):
    x = torch.randn(4, 64, device=cuda_device)
    kat.KAT_Group()(x)
    maps = open("/proc/self/maps").read()
    assert "libkat_rational.so" in maps


@pytest.mark.parametrize("name", case_names())
def test_golden_case(name, cuda_device):
    c = load_case(name)
    out = run_module(c["x"], c["grad_out"], c["w_num"], c["w_den"], c["G"], c["layout"],
                     cuda_device, TORCH_DTYPES[c["dtype"]])
    assert out[0].dtype == TORCH_DTYPES[c["dtype"]] and out[0].shape == c["x"].shape
    oracle = oracle_for(c["x"], c["grad_out"], c["w_num"], c["w_den"], c["dims"], c["G"])
    assert_parity(out, (c["y"], c["dx"]), oracle, c["dtype"], name)
    # Distance to the reference's own fp32 coefficient gradients (which carry fp32
    # summation error of their own): 1e-4 of the gradient scale.
    for got, ref, mag in ((out[2], c["d_num"], oracle[2]["d_num_mag"].sum(0, keepdims=True)),
                          (out[3], c["d_den"], oracle[2]["d_den_mag"])):
        assert_coef_grads(got, ref.numpy(), mag, f"{name}/grads vs reference fp32")


@pytest.mark.parametrize("name", ["identity_blc_f32", "identity_nchw_f32", "mode_identity"])
def test_identity_is_exact(name, cuda_device):
    c = load_case(name)
    y, dx, dn, dd = run_module(c["x"], c["grad_out"], c["w_num"], c["w_den"], c["G"],
                               c["layout"], cuda_device)
    assert torch.equal(y.cpu(), c["x"])
    assert torch.equal(dx.cpu(), c["grad_out"])
    assert torch.count_nonzero(dd) == 0


def _random_case(shape, groups, layout, dtype, seed=11, x_std=1.5, coef_std=0.3):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(*shape, generator=g) * x_std).to(TORCH_DTYPES[dtype]).float()
    gy = torch.randn(*shape, generator=g).to(TORCH_DTYPES[dtype]).float()
    wn = torch.randn(1, 6, generator=g) * coef_std
    wd = torch.randn(groups, 4, generator=g) * coef_std
    return x, gy, wn, wd


def _dims(shape, layout):
    if layout == "nchw":
        return shape[0], shape[1], shape[2] * shape[3]
    return int(np.prod(shape)) // shape[-1], shape[-1], 1


EDGE_SHAPES = [
    # shape, groups, layout, dtype
    ((3, 5, 36), 12, "blc", "f32"),        # group width 3: scalar path
    ((2, 7, 36), 12, "blc", "bf16"),
    ((4, 768), 64, "blc", "bf16"),         # [B, C], 12-wide groups
    ((2, 3, 8192), 64, "blc", "f32"),      # several column blocks per row
    ((2, 3, 8192), 16, "blc", "f16"),
    ((1, 1, 8), 8, "blc", "f32"),          # one element per group
    ((5, 1000, 24), 3, "blc", "f32"),      # many rows, 8-wide groups
    ((3, 16, 7, 7), 8, "nchw", "f32"),     # 7x7: odd spatial size
    ((2, 32, 5, 3), 4, "nchw", "bf16"),
    ((2, 6, 1, 1), 3, "nchw", "f16"),
    ((257, 3, 96), 8, "blc", "f16"),
    # short, wide problems: the cp.async backward takes 512-column tiles (at 128 columns more
    # column blocks than blocks, several ring refills per block)
    ((4, 64, 56, 56), 8, "nchw", "f32"),
    ((4, 262144), 8, "blc", "bf16"),
    # blocks aligned to column blocks, unevenly (16, 8 and 6 column blocks on 148 blocks)
    ((16, 16384), 8, "blc", "bf16"),
    ((37, 8192), 8, "blc", "bf16"),
    ((300, 6144), 16, "blc", "f16"),
]


@pytest.mark.parametrize("shape,groups,layout,dtype", EDGE_SHAPES)
def test_edge_shapes(shape, groups, layout, dtype, cuda_device):
    x, gy, wn, wd = _random_case(shape, groups, layout, dtype)
    out = run_module(x, gy, wn, wd, groups, layout, cuda_device, TORCH_DTYPES[dtype])
    oracle = oracle_for(x, gy, wn, wd, _dims(shape, layout), groups)
    assert_parity(out, None, oracle, dtype, f"{shape}/{groups}/{dtype}")


def test_empty_input(cuda_device):
    m = kat.KAT_Group(num_groups=4).to(cuda_device)
    x = torch.empty(0, 5, 16, device=cuda_device, requires_grad=True)
    y = m(x)
    assert y.shape == (0, 5, 16)
    y.backward(torch.empty_like(y))
    assert torch.count_nonzero(m.weight_numerator.grad) == 0
    assert torch.count_nonzero(m.weight_denominator.grad) == 0
    assert x.grad.shape == x.shape


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_misaligned_and_strided_inputs(dtype, cuda_device):
    """A 1-element offset defeats 16-byte vectors (scalar path); a transposed view is
    made contiguous by the wrapper."""
    shape, groups = (6, 4, 64), 8
    x, gy, wn, wd = _random_case(shape, groups, "blc", dtype)
    tdt = TORCH_DTYPES[dtype]
    base = torch.empty(x.numel() + 1, device=cuda_device, dtype=tdt)
    base[1:] = x.reshape(-1).to(cuda_device, tdt)
    xm = base[1:].view(shape)
    assert xm.data_ptr() % 16 != 0
    y = kat.rational_fwd_cuda(xm, wn.repeat(groups, 1).to(cuda_device), wd.to(cuda_device), groups)
    y_ref = kat.rational_fwd_cuda(x.to(cuda_device, tdt), wn.repeat(groups, 1).to(cuda_device),
                                  wd.to(cuda_device), groups)
    assert torch.equal(y, y_ref)
    xt = x.to(cuda_device, tdt).transpose(0, 1).contiguous().transpose(0, 1)
    assert not xt.is_contiguous()
    y_t = kat.rational_fwd_cuda(xt, wn.repeat(groups, 1).to(cuda_device), wd.to(cuda_device),
                                groups)
    assert torch.equal(y_t, y_ref)


def test_input_without_grad_skips_dx(cuda_device):
    x, gy, wn, wd = _random_case((4, 5, 64), 8, "blc", "f32")
    m = kat.KAT_Group(num_groups=8).to(cuda_device)
    with torch.no_grad():
        m.weight_numerator.copy_(wn)
        m.weight_denominator.copy_(wd)
    y = m(x.to(cuda_device))
    y.backward(gy.to(cuda_device))
    _, _, b = oracle_for(x, gy, wn, wd, _dims((4, 5, 64), "blc"), 8)
    assert_coef_grads(m.weight_numerator.grad, b["d_num"].sum(0, keepdims=True),
                      b["d_num_mag"].sum(0, keepdims=True), "no-dx/d_num")
    assert_coef_grads(m.weight_denominator.grad, b["d_den"], b["d_den_mag"], "no-dx/d_den")


def test_autocast_casts_to_fp32(cuda_device):
    m = kat.KAT_Group(num_groups=8).to(cuda_device)
    x = torch.randn(2, 3, 64, device=cuda_device, dtype=torch.bfloat16)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y = m(x)
    assert y.dtype == torch.float32
    y_plain = m(x)
    assert y_plain.dtype == torch.bfloat16


def test_nan_and_pole_classes(cuda_device):
    """NaN inputs propagate to y, dx and their group's coefficient gradients; huge inputs
    and poles give the same inf/NaN classes as the float64 oracle."""
    shape, groups = (2, 3, 32), 4
    x, gy, wn, wd = _random_case(shape, groups, "blc", "f32")
    x = x.clone()
    x[0, 1, 3] = float("nan")      # group 0
    out = run_module(x, gy, wn, wd, groups, "blc", cuda_device)
    oracle = oracle_for(x, gy, wn, wd, _dims(shape, "blc"), groups)
    assert torch.isnan(out[0][0, 1, 3]) and torch.isnan(out[1][0, 1, 3])
    assert torch.isnan(out[3][0]).all() and torch.isfinite(out[3][1:]).all()
    assert_elementwise(out[0], oracle[0], oracle[1], "f32", "nan/y")
    assert_elementwise(out[1], oracle[2]["dx"], oracle[2]["dx_mag"], "f32", "nan/dx")


def test_determinism(cuda_device):
    """Coefficient gradients and dx are bit-identical over repeated runs."""
    x, gy, wn, wd = _random_case((64, 197, 768), 8, "blc", "bf16", x_std=1.0)
    xd, gd = x.to(cuda_device, torch.bfloat16), gy.to(cuda_device, torch.bfloat16)
    n = wn.repeat(8, 1).to(cuda_device)
    d = wd.to(cuda_device)
    first = kat.rational_bwd_cuda(gd, xd, n, d, 8)
    for _ in range(10):
        again = kat.rational_bwd_cuda(gd, xd, n, d, 8)
        for a, b in zip(first, again):
            assert torch.equal(a, b)


def test_workspace_too_small_is_rejected(cuda_device):
    x = torch.randn(64, 256, device=cuda_device)
    gy = torch.randn_like(x)
    dx = torch.empty_like(x)
    n = torch.randn(4, 6, device=cuda_device)
    d = torch.randn(4, 4, device=cuda_device)
    dn = torch.empty(4, 6, device=cuda_device)
    dd = torch.empty(4, 4, device=cuda_device)
    lib = _native.lib()
    need = ctypes.c_size_t(0)
    assert lib.kat_rational_bwd_workspace_size(64, 256, 1, 4, 0, cuda_device.index or 0,
                                               ctypes.byref(need)) == 0
    assert need.value > 0
    ws = torch.empty(need.value, dtype=torch.uint8, device=cuda_device)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    st = lib.kat_rational_bwd(x.data_ptr(), gy.data_ptr(), dx.data_ptr(), n.data_ptr(),
                              d.data_ptr(), dn.data_ptr(), dd.data_ptr(), ws.data_ptr(),
                              need.value - 8, 64, 256, 1, 4, 0, stream)
    assert st == _native.KAT_ERR_WORKSPACE
    st = lib.kat_rational_bwd(x.data_ptr(), gy.data_ptr(), dx.data_ptr(), n.data_ptr(),
                              d.data_ptr(), dn.data_ptr(), dd.data_ptr(), ws.data_ptr(),
                              need.value, 64, 256, 1, 4, 0, stream)
    assert st == _native.KAT_OK
    torch.cuda.synchronize()
