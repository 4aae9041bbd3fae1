"""rat_cuda (abs-after-sum formula) on the GPU against the oracle.

The primary bars are this library's: fp32 y/dx within 1e-6 of the float64 oracle
(condition-aware: relative to max(|ref|, magnitude of the terms)), 16-bit outputs within one
ulp of the rounded fp32 oracle, coefficient gradients within 1e-4 relative, bit-identical
repeats — on the golden cases made from the reference's own formula code, vector and scalar
paths, NCHW through the C ABI and the ViT-B MLP-hidden size.

The reference suite's checks (tests/test_correctness.py) are mirrored too: gradcheck in
float64 and identity coefficients as they are; its absolute bars (forward 1e-5, backward
1e-4, bf16 inputs 5e-3) are applied relative to max(1, magnitude of the terms), because two
fp32 evaluations in different operation orders (fma Horner here, separate multiply and add
in its PyTorch definition) differ in proportion to the size of the terms, and a bf16 input
rounding moves y in proportion to it as well."""

import ctypes
import json
import os

import numpy as np
import pytest
import torch

import rational_kat_cu_b200 as kat
from oracle import rat_torch_oracle as rat
from rational_kat_cu_b200 import _native
from tolerances import assert_coef_grads, assert_elementwise

pytestmark = pytest.mark.gpu

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
MANIFEST = json.load(open(os.path.join(HERE, "rat_cases.json")))["cases"]
DT = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


def golden(name):
    data = np.load(os.path.join(HERE, "golden_rat.npz"))
    meta = next(c for c in MANIFEST if c["name"] == name)
    return meta, {k: torch.from_numpy(data[f"{name}/{k}"]) for k in
                  ("x", "gy", "a", "b", "y", "dx", "da", "db")}


def run(x, a, b, gy, dev):
    xd = x.detach().to(dev).requires_grad_(True)
    ad = a.detach().to(dev).requires_grad_(True)
    bd = b.detach().to(dev).requires_grad_(True)
    y = kat.rat_cuda(xd, ad, bd)
    y.backward(gy.to(dev, dtype=y.dtype))
    return y.detach().cpu(), xd.grad.cpu(), ad.grad.cpu(), bd.grad.cpu()


def check(x, a, b, gy, y, dx, da, db, dtype, name, db_ok=True):
    """Kernel outputs against the float64 oracle (and the fp32 oracle rounded to a 16-bit
    output dtype)."""
    y64, dx64, da64, db64 = rat.rat_forward_backward(x.float(), a, b, gy.float(),
                                                     compute_dtype=torch.float64,
                                                     grouped_numerator_grad=True)
    ymag, dxmag, nmag, dmag = rat.rat_magnitudes(x.float(), a, b, gy.float())
    if dtype == "f32":
        assert_elementwise(y, y64, ymag, "f32", f"{name}/y")
        assert_elementwise(dx, dx64, dxmag, "f32", f"{name}/dx")
    else:
        y32, dx32, _, _ = rat.rat_forward_backward(x.float(), a, b, gy.float())
        assert_elementwise(y, y64, ymag, dtype, f"{name}/y", ref_rounded=y32.to(DT[dtype]))
        assert_elementwise(dx, dx64, dxmag, dtype, f"{name}/dx", ref_rounded=dx32.to(DT[dtype]))
    assert_coef_grads(da, da64.sum(0), nmag.sum(0), f"{name}/da")
    if db_ok:
        assert_coef_grads(db, db64, dmag, f"{name}/db")


@pytest.mark.parametrize("name", [c["name"] for c in MANIFEST])
def test_golden_cases(name, cuda_device):
    meta, c = golden(name)
    dt = meta["input_dtype"]
    x = c["x"].to(DT[dt])
    gy = c["gy"].to(DT[dt])
    y, dx, da, db = run(x, c["a"], c["b"], gy, cuda_device)
    check(x, c["a"], c["b"], gy, y, dx, da, db, dt, name)
    if dt == "f32":
        # against the reference's own fp32 numbers, at the reference suite's bars (scaled)
        ymag, dxmag, _, _ = rat.rat_magnitudes(x, c["a"], c["b"], gy)
        assert bool(((y - c["y"]).abs() <= 1e-5 * ymag.float().clamp(min=1.0)).all())
        assert bool(((dx - c["dx"]).abs() <= 1e-4 * dxmag.float().clamp(min=1.0)).all())
        assert (da - c["da"]).abs().max() < 1e-4 * max(1.0, c["da"].abs().max().item())
        if meta["db_comparable"]:
            assert (db - c["db"]).abs().max() < 1e-4 * max(1.0, c["db"].abs().max().item())


@pytest.mark.parametrize("N,D,G", [(4, 64, 8), (32, 256, 8), (128, 768, 8), (1, 32, 4)])
def test_forward_correctness(N, D, G, cuda_device):
    torch.manual_seed(42)
    x = torch.randn(N, D)
    a = torch.randn(6)
    b = torch.randn(G, 4)
    y = kat.rat_cuda(x.to(cuda_device), a.to(cuda_device), b.to(cuda_device)).cpu()
    ref = rat.rat_forward_grouped(x, a.view(1, 6).expand(G, 6), b)
    ymag = rat.rat_magnitudes(x, a, b, torch.ones_like(x))[0].float()
    assert y.shape == x.shape
    assert bool(((y - ref).abs() <= 1e-5 * ymag.clamp(min=1.0)).all())


@pytest.mark.parametrize("N,D,G", [(4, 64, 1), (8, 256, 1), (4, 64, 4), (8, 128, 8)])
def test_gradcheck_float64(N, D, G, cuda_device):
    torch.manual_seed(42)
    x = torch.randn(N, D, device=cuda_device, dtype=torch.float64, requires_grad=True)
    a = torch.randn(6, device=cuda_device, dtype=torch.float64, requires_grad=True)
    b = torch.randn(G, 4, device=cuda_device, dtype=torch.float64, requires_grad=True)
    assert torch.autograd.gradcheck(kat.rat_cuda, (x, a, b), eps=1e-4, atol=1e-3, rtol=1e-3,
                                    raise_exception=True)


def test_backward_vs_autograd(cuda_device):
    torch.manual_seed(42)
    N, D, G = 32, 256, 8
    x, a, b = torch.randn(N, D), torch.randn(6), torch.randn(G, 4)
    gy = torch.randn(N, D)
    y, dx, da, db = run(x, a, b, gy, cuda_device)
    _, dx_r, da_r, db_r = rat.rat_forward_backward(x, a, b, gy)
    dxmag = rat.rat_magnitudes(x, a, b, gy)[1].float()
    assert bool(((dx - dx_r).abs() <= 1e-4 * dxmag.clamp(min=1.0)).all())
    for name, got, want in (("da", da, da_r), ("db", db, db_r)):
        assert (got - want).abs().max().item() < 1e-4 * max(1.0, want.abs().max().item()), name


def test_bf16_inputs_track_fp32(cuda_device):
    torch.manual_seed(42)
    N, D, G = 16, 128, 8
    x, a, b = torch.randn(N, D), torch.randn(6), torch.randn(G, 4)
    d = cuda_device
    out32 = kat.rat_cuda(x.to(d), a.to(d), b.to(d)).cpu()
    xb, ab, bb = x.bfloat16(), a.bfloat16(), b.bfloat16()
    out16 = kat.rat_cuda(xb.to(d), ab.to(d), bb.to(d)).cpu()
    assert out16.dtype == torch.bfloat16
    # the kernel on the rounded inputs: one bf16 ulp of the fp32 oracle on the same inputs
    y64, _, _, _ = rat.rat_forward_backward(xb.float(), ab.float(), bb.float(), torch.ones(N, D),
                                            compute_dtype=torch.float64)
    y32, _, _, _ = rat.rat_forward_backward(xb.float(), ab.float(), bb.float(), torch.ones(N, D))
    mag = rat.rat_magnitudes(xb.float(), ab.float(), bb.float(), torch.ones(N, D))[0]
    assert_elementwise(out16, y64, mag, "bf16", "bf16 inputs", ref_rounded=y32.bfloat16())
    # against the fp32 run: the reference suite's 5e-3 plus what rounding x, a and b to bf16
    # (relative 2^-9 each) can move y by
    ymag = rat.rat_magnitudes(x, a, b, torch.ones(N, D))[0].float()
    assert bool(((out32 - out16.float()).abs() <= 5e-3 + 2.0 ** -5 * ymag).all())


def test_autocast_runs_in_fp32(cuda_device):
    torch.manual_seed(1)
    x = torch.randn(8, 64, device=cuda_device, requires_grad=True)
    a = torch.randn(6, device=cuda_device, requires_grad=True)
    b = torch.randn(8, 4, device=cuda_device, requires_grad=True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y = kat.rat_cuda(x.to(torch.bfloat16), a, b)
    assert y.dtype == torch.float32
    y.sum().backward()
    assert a.grad.shape == (6,) and b.grad.shape == (8, 4)


def test_identity_coefficients(cuda_device):
    torch.manual_seed(42)
    N, D, G = 8, 128, 8
    x = torch.randn(N, D, device=cuda_device)
    a = torch.zeros(6, device=cuda_device)
    a[1] = 1.0
    b = torch.zeros(G, 4, device=cuda_device)
    out = kat.rat_cuda(x, a, b)
    assert torch.equal(out, x)
    # +1 sign at D = 0: d b_j = -sum go * x * x^(j+1)
    gy = torch.randn(N, D, device=cuda_device)
    _, _, _, db = run(x.cpu(), a.cpu(), b.cpu(), gy.cpu(), cuda_device)
    xg = x.double().cpu().reshape(N, G, D // G)
    gg = gy.double().cpu().reshape(N, G, D // G)
    want = torch.stack([-(gg * xg * xg ** (j + 1)).sum(dim=(0, 2)) for j in range(4)], dim=1)
    assert_coef_grads(db, want, want.abs() + 1e-30, "identity/db")


@pytest.mark.parametrize("N,D,G,dt", [
    (257, 96, 8, "bf16"),    # 12-wide groups: 4-element vectors
    (33, 36, 12, "f32"),     # 3-wide groups: scalar path
    (64, 3072, 8, "f16"),
    (500, 768, 64, "bf16"),
    (300, 8192, 16, "f32"),
])
def test_shapes_and_dtypes(N, D, G, dt, cuda_device):
    g = torch.Generator().manual_seed(N + D + G)
    x = (torch.randn(N, D, generator=g) * 2.0).to(DT[dt])
    gy = torch.randn(N, D, generator=g).to(DT[dt])
    a = torch.randn(6, generator=g) * 0.5
    b = torch.randn(G, 4, generator=g) * 0.5
    y, dx, da, db = run(x, a, b, gy, cuda_device)
    assert y.dtype == DT[dt] and dx.dtype == DT[dt]
    check(x, a, b, gy, y, dx, da.view(6), db, dt, f"rat_{N}x{D}_g{G}_{dt}")


def test_nchw_through_c_abi(cuda_device):
    """kat_rational_fwd_formula / _bwd_formula with inner = H*W (NCHW) against the oracle on
    the channels-last permutation."""
    B, C, H, W, G = 3, 32, 7, 7, 4
    g = torch.Generator().manual_seed(9)
    x = torch.randn(B, C, H, W, generator=g)
    gy = torch.randn(B, C, H, W, generator=g)
    a = torch.randn(6, generator=g)
    b = torch.randn(G, 4, generator=g)
    d = cuda_device
    lib = _native.lib()
    xd, gd = x.to(d), gy.to(d)
    num = a.view(1, 6).repeat(G, 1).to(d)
    den = b.to(d)
    y = torch.empty_like(xd)
    dx = torch.empty_like(xd)
    dn = torch.empty(G, 6, device=d)
    dd = torch.empty(G, 4, device=d)
    need = ctypes.c_size_t()
    _native.check("ws", lib.kat_rational_bwd_workspace_size(B, C, H * W, G, 0, d.index,
                                                            ctypes.byref(need)))
    ws = torch.empty(max(need.value, 16), dtype=torch.uint8, device=d)
    s = ctypes.c_void_p(torch.cuda.current_stream(d).cuda_stream)
    _native.check("fwd", lib.kat_rational_fwd_formula(xd.data_ptr(), y.data_ptr(), num.data_ptr(),
                                                      den.data_ptr(), B, C, H * W, G, 0,
                                                      _native.KAT_FORMULA_ABS_SUM, s))
    _native.check("bwd", lib.kat_rational_bwd_formula(
        xd.data_ptr(), gd.data_ptr(), dx.data_ptr(), num.data_ptr(), den.data_ptr(),
        dn.data_ptr(), dd.data_ptr(), ws.data_ptr(), ws.numel(), B, C, H * W, G, 0,
        _native.KAT_FORMULA_ABS_SUM, s))
    torch.cuda.synchronize(d)
    to_blc = lambda t: t.permute(0, 2, 3, 1).reshape(B * H * W, C)
    check(to_blc(x), a, b, to_blc(gy), to_blc(y.cpu()), to_blc(dx.cpu()), dn.cpu().sum(0), dd.cpu(),
          "f32", "rat_nchw")
    # the same call with KAT_FORMULA_KAT is the KAT activation (not the abs-after-sum one)
    y2 = torch.empty_like(xd)
    _native.check("fwd", lib.kat_rational_fwd_formula(xd.data_ptr(), y2.data_ptr(), num.data_ptr(),
                                                      den.data_ptr(), B, C, H * W, G, 0,
                                                      _native.KAT_FORMULA_KAT, s))
    y3 = kat.rational_fwd_cuda_2d(xd, num, den, G)
    torch.cuda.synchronize(d)
    assert torch.equal(y2, y3)


def test_coefficient_gradients_bit_reproducible(cuda_device):
    g = torch.Generator().manual_seed(5)
    x = torch.randn(4096, 768, generator=g).to(cuda_device, torch.bfloat16)
    gy = torch.randn(4096, 768, generator=g).to(cuda_device, torch.bfloat16)
    a = torch.randn(6, generator=g).to(cuda_device)
    b = torch.randn(8, 4, generator=g).to(cuda_device)
    outs = []
    for _ in range(5):
        aa = a.clone().requires_grad_(True)
        bb = b.clone().requires_grad_(True)
        kat.rat_cuda(x, aa, bb).backward(gy)
        outs.append((aa.grad.clone(), bb.grad.clone()))
    for o in outs[1:]:
        assert torch.equal(o[0], outs[0][0]) and torch.equal(o[1], outs[0][1])


def test_vitb_hidden_size_bf16(cuda_device):
    """[128*197, 3072] bf16: elementwise outputs on sampled rows against the oracle; the
    coefficient gradients over the full tensor against a float64 torch evaluation of the same
    formula (on the GPU, in row chunks)."""
    N, D, G = 128 * 197, 3072, 8
    d = cuda_device
    gen = torch.Generator(device=d).manual_seed(0)
    x = torch.randn(N, D, generator=gen, device=d).to(torch.bfloat16)
    gy = torch.randn(N, D, generator=gen, device=d).to(torch.bfloat16)
    a = torch.randn(6, generator=torch.Generator().manual_seed(3)) * 0.5
    b = torch.randn(G, 4, generator=torch.Generator().manual_seed(4)) * 0.5
    aa = a.to(d).requires_grad_(True)
    bb = b.to(d).requires_grad_(True)
    xr = x.detach().requires_grad_(True)
    y = kat.rat_cuda(xr, aa, bb)
    y.backward(gy)
    rows = torch.cat([torch.arange(0, 256), torch.arange(N - 256, N)])
    xs, gs = x[rows].cpu(), gy[rows].cpu()
    y64, dx64, _, _ = rat.rat_forward_backward(xs.float(), a, b, gs.float(),
                                               compute_dtype=torch.float64)
    y32, dx32, _, _ = rat.rat_forward_backward(xs.float(), a, b, gs.float())
    ymag, dxmag, _, _ = rat.rat_magnitudes(xs.float(), a, b, gs.float())
    assert_elementwise(y.detach()[rows].cpu(), y64, ymag, "bf16", "vitb/y",
                       ref_rounded=y32.to(torch.bfloat16))
    assert_elementwise(xr.grad[rows].cpu(), dx64, dxmag, "bf16", "vitb/dx",
                       ref_rounded=dx32.to(torch.bfloat16))
    da64 = torch.zeros(6, dtype=torch.float64, device=d)
    db64 = torch.zeros(G, 4, dtype=torch.float64, device=d)
    nm = torch.zeros(6, dtype=torch.float64, device=d)
    dm = torch.zeros(G, 4, dtype=torch.float64, device=d)
    for r0 in range(0, N, 4096):
        xc, gc = x[r0:r0 + 4096].double(), gy[r0:r0 + 4096].double()
        _, _, da_c, db_c = rat.rat_forward_backward(xc, a.to(d), b.to(d), gc,
                                                    compute_dtype=torch.float64)
        _, _, nm_c, dm_c = rat.rat_magnitudes(xc, a.to(d), b.to(d), gc)
        da64 += da_c
        db64 += db_c
        nm += nm_c.sum(0)
        dm += dm_c
    assert_coef_grads(aa.grad.cpu(), da64.cpu(), nm.cpu(), "vitb/da")
    assert_coef_grads(bb.grad.cpu(), db64.cpu(), dm.cpu(), "vitb/db")
