"""The benchmark workloads at full size on the GPU, checked element by element against the
float64 oracle (row chunks, so host memory stays bounded), plus the coefficient gradients,
and size-independent properties at up to 2^31 elements (64-bit indexing).

  kat_group_f32        x[8,197,768] fp32 'gelu'       (also vs the golden reference sample)
  kat_group_vitb_bf16  x[128,197,3072] bf16 'gelu'+N(0,0.01)
  kat_group2d_f32      x[64,256,56,56] fp32 NCHW 'identity'  (y == x, dx == grad_out exactly)
  sweep points         x[N/C, C], C in {768, 3072, 8192}, G in {8, 16, 64}
"""

import numpy as np
import pytest
import torch

import rational_kat_cu_b200 as kat
from golden_data import load_cfg1
from oracle import c_oracle
from rational_kat_cu_b200 import workloads
from tolerances import assert_coef_grads, assert_elementwise

pytestmark = pytest.mark.gpu

OUT_NAME = {"f32": "f32", "bf16": "bf16", "f16": "f16"}


def run_workload(w, device, on_gpu_inputs=False):
    x, gy = w.inputs(device if on_gpu_inputs else None)
    wn, wd = w.coefficients()
    cls = kat.KAT_Group2D if w.layout == "nchw" else kat.KAT_Group
    mod = cls(num_groups=w.groups, mode="gelu").to(device)
    with torch.no_grad():
        mod.weight_numerator.copy_(wn)
        mod.weight_denominator.copy_(wd)
    xd = x.detach().to(device).requires_grad_(True)
    y = mod(xd)
    y.backward(gy.to(device))
    torch.cuda.synchronize()
    return x, gy, wn, wd, y.detach(), xd.grad, mod.weight_numerator.grad, mod.weight_denominator.grad


def check_against_oracle(w, x, gy, wn, wd, y, dx, dn, dd, chunk_rows=2048):
    """Elementwise y, dx and the coefficient gradients against the float64 oracle."""
    batch, channels, inner = w.dims()
    row = channels * inner
    xf = x.reshape(batch, row)
    gf = gy.reshape(batch, row)
    yf = y.reshape(batch, row)
    dxf = dx.reshape(batch, row)
    tot = {k: 0.0 for k in ("d_num", "d_den", "d_num_mag", "d_den_mag")}
    tdt = workloads.DTYPES[w.dtype]
    for r0 in range(0, batch, chunk_rows):
        r1 = min(batch, r0 + chunk_rows)
        xs = xf[r0:r1].float().reshape(-1).numpy()
        gs = gf[r0:r1].float().reshape(-1).numpy()
        dims = (r1 - r0, channels, inner)
        y64, ymag = c_oracle.forward(xs, wn.numpy(), wd.numpy(), dims, w.groups)
        b = c_oracle.backward(xs, gs, wn.numpy(), wd.numpy(), dims, w.groups)
        ys = yf[r0:r1].cpu().float().reshape(-1)
        dxs = dxf[r0:r1].cpu().float().reshape(-1)
        if w.dtype == "f32":
            assert_elementwise(ys, y64, ymag, "f32", f"{w.name}/y rows {r0}:{r1}")
            assert_elementwise(dxs, b["dx"], b["dx_mag"], "f32", f"{w.name}/dx rows {r0}:{r1}")
        else:
            y32 = torch.from_numpy(y64).float()
            d32 = torch.from_numpy(b["dx"]).float()
            assert_elementwise(ys, y64, ymag, w.dtype, f"{w.name}/y rows {r0}:{r1}",
                               ref_rounded=y32.to(tdt).float())
            assert_elementwise(dxs, b["dx"], b["dx_mag"], w.dtype,
                               f"{w.name}/dx rows {r0}:{r1}", ref_rounded=d32.to(tdt).float())
        for k in tot:
            tot[k] = tot[k] + b[k]
    assert_coef_grads(dn, tot["d_num"].sum(0, keepdims=True),
                      tot["d_num_mag"].sum(0, keepdims=True), f"{w.name}/d_num")
    assert_coef_grads(dd, tot["d_den"], tot["d_den_mag"], f"{w.name}/d_den")


def test_kat_group_f32_full(cuda_device):
    w = workloads.kat_group_f32()
    x, gy, wn, wd, y, dx, dn, dd = run_workload(w, cuda_device)
    check_against_oracle(w, x, gy, wn, wd, y.cpu(), dx.cpu(), dn, dd)
    g = load_cfg1()
    idx = g["index"]
    _, ymag = c_oracle.forward(x.reshape(-1).numpy(), wn.numpy(), wd.numpy(), w.dims(), w.groups)
    b = c_oracle.backward(x.reshape(-1).numpy(), gy.reshape(-1).numpy(), wn.numpy(), wd.numpy(),
                          w.dims(), w.groups)
    assert_elementwise(y.reshape(-1).cpu()[idx], g["y_sample"], ymag[idx], "f32",
                       "cfg1/y vs reference")
    assert_elementwise(dx.reshape(-1).cpu()[idx], g["dx_sample"], b["dx_mag"][idx], "f32",
                       "cfg1/dx vs reference")
    assert_coef_grads(dn, g["d_num"], b["d_num_mag"].sum(0, keepdims=True),
                      "cfg1/d_num vs reference fp32")
    assert_coef_grads(dd, g["d_den"], b["d_den_mag"], "cfg1/d_den vs reference fp32")


def test_kat_group_vitb_bf16_full(cuda_device):
    w = workloads.kat_group_vitb_bf16()
    x, gy, wn, wd, y, dx, dn, dd = run_workload(w, cuda_device)
    check_against_oracle(w, x, gy, wn, wd, y.cpu(), dx.cpu(), dn, dd)


def test_kat_group2d_f32_full(cuda_device):
    w = workloads.kat_group2d_f32()
    x, gy, wn, wd, y, dx, dn, dd = run_workload(w, cuda_device)
    assert torch.equal(y.cpu(), x)
    assert torch.equal(dx.cpu(), gy)
    assert torch.count_nonzero(dd) == 0
    b_num = 0.0
    batch, channels, inner = w.dims()
    for r0 in range(0, batch, 16):
        xs = x[r0:r0 + 16].reshape(-1).numpy()
        gs = gy[r0:r0 + 16].reshape(-1).numpy()
        b = c_oracle.backward(xs, gs, wn.numpy(), wd.numpy(), (xs.size // (channels * inner),
                              channels, inner), w.groups, want_dx=False)
        b_num = b_num + np.concatenate([b["d_num"], b["d_num_mag"]], axis=1)
    assert_coef_grads(dn, b_num[:, :6].sum(0, keepdims=True), b_num[:, 6:].sum(0, keepdims=True),
                      "cfg3/d_num")


SWEEP = [
    (768, 8, 1 << 20, "f32"),
    (3072, 16, 1 << 22, "bf16"),
    (8192, 64, 1 << 22, "f16"),
    (768, 64, 1 << 24, "bf16"),
    (8192, 8, 1 << 24, "f32"),
    (3072, 64, 1 << 23, "f16"),
]


@pytest.mark.parametrize("channels,groups,numel,dtype", SWEEP)
def test_sweep_points(channels, groups, numel, dtype, cuda_device):
    w = workloads.sweep(channels, groups, numel, dtype)
    x, gy, wn, wd, y, dx, dn, dd = run_workload(w, cuda_device, on_gpu_inputs=True)
    check_against_oracle(w, x.cpu(), gy.cpu(), wn, wd, y.cpu(), dx.cpu(), dn, dd)


def test_beyond_int32_elements(cuda_device):
    """2^31 + C elements of bf16 (64-bit offsets): identity coefficients make y == x and
    dx == grad_out exactly everywhere; random coefficients are then checked on the rows
    past element 2^31 against the float64 oracle."""
    C, G = 3072, 8
    rows = (1 << 31) // C + 2
    gen = torch.Generator(device=cuda_device).manual_seed(0)
    x = torch.randn(rows, C, generator=gen, device=cuda_device, dtype=torch.float32).to(
        torch.bfloat16)
    gy = torch.randn(rows, C, generator=gen, device=cuda_device, dtype=torch.float32).to(
        torch.bfloat16)
    assert x.numel() > (1 << 31)
    ident = kat.KAT_Group(num_groups=G, mode="identity")
    n = ident.weight_numerator.detach().repeat(G, 1).to(cuda_device)
    d = ident.weight_denominator.detach().to(cuda_device)
    y = kat.rational_fwd_cuda(x, n, d, G)
    assert torch.equal(y, x)
    del y
    dx, dn, dd = kat.rational_bwd_cuda(gy, x, n, d, G)
    assert torch.equal(dx, gy)
    del dx
    assert torch.count_nonzero(dd) == 0
    # d_num[g, 0] = sum of grad_out over group g; check it against a float64 sum.
    ref0 = torch.sum(gy.view(rows, G, C // G), dim=(0, 2), dtype=torch.float64)
    np.testing.assert_allclose(dn[:, 0].double().cpu().numpy(), ref0.cpu().numpy(),
                               rtol=1e-4, atol=1e-2)
    # Random coefficients: the tail rows, beyond 32-bit element offsets.
    w = workloads.sweep(C, G, C, "bf16")
    wn, wd = w.coefficients()
    y = kat.rational_fwd_cuda(x, wn.repeat(G, 1).to(cuda_device), wd.to(cuda_device), G)
    tail = slice(rows - 3, rows)
    xs = x[tail].float().reshape(-1).cpu().numpy()
    y64, ymag = c_oracle.forward(xs, wn.numpy(), wd.numpy(), (3, C, 1), G)
    ys = y[tail].float().reshape(-1).cpu()
    assert_elementwise(ys, y64, ymag, "bf16", "tail/y",
                       ref_rounded=torch.from_numpy(y64).float().to(torch.bfloat16).float())
