"""KAT_Group / KAT_Group2D pass their [1, 6] numerator to the kernels as one shared row
(KAT_SHARED_NUMERATOR) instead of repeating it per group: against the reference-contract
Functions (RationalCUDA1DGroup / RationalCUDA2D on weight_numerator.repeat(G, 1), whose d_n
[G, 6] torch then sums), y, d_input and d_denominator must be bit-identical, and d_numerator
[1, 6] must equal the float64 sum over groups of the per-group gradients rounded once, and be
bit-identical from run to run."""

import pytest
import torch

import rational_kat_cu_b200 as kat
from rational_kat_cu_b200.rational_cuda import KatGroupFunction, RationalCUDA1DGroup, RationalCUDA2D

pytestmark = pytest.mark.gpu

CASES = [
    ((4, 197, 768), 8, torch.bfloat16, False),
    ((6, 64), 4, torch.float32, False),
    ((3, 5, 36), 12, torch.float16, False),
    ((2, 64, 7, 7), 8, torch.float32, True),
    ((2, 32, 56, 56), 8, torch.bfloat16, True),
    ((64, 3072), 64, torch.bfloat16, False),
]


@pytest.mark.parametrize("shape,G,dtype,nchw", CASES)
def test_shared_row_matches_repeated_numerator(shape, G, dtype, nchw):
    g = torch.Generator(device="cpu").manual_seed(3)
    x = (torch.randn(*shape, generator=g) * 1.3).to(dtype).cuda()
    gy = torch.randn(*shape, generator=g).to(dtype).cuda()
    wn = (torch.randn(1, 6, generator=g) * 0.4).cuda()
    wd = (torch.randn(G, 4, generator=g) * 0.4).cuda()

    def run(shared):
        xi = x.clone().requires_grad_(True)
        n = wn.clone().requires_grad_(True)
        d = wd.clone().requires_grad_(True)
        if shared:
            y = KatGroupFunction.apply(xi, n, d, G, nchw)
        else:
            fn = RationalCUDA2D if nchw else RationalCUDA1DGroup
            y = fn.apply(xi, n.repeat(G, 1), d, G)
        y.backward(gy)
        return y.detach(), xi.grad, n.grad, d.grad

    ys, dxs, dns, dds = run(True)
    yr, dxr, _, ddr = run(False)
    assert torch.equal(ys, yr) and torch.equal(dxs, dxr) and torch.equal(dds, ddr)
    # d_numerator: the per-group gradients (the reference contract, [G, 6]) summed in float64
    per_group = RationalCUDA2D if nchw else RationalCUDA1DGroup
    xi = x.clone()
    _, d_n_g, _ = (kat.rational_bwd_cuda_2d if nchw else kat.rational_bwd_cuda)(
        gy, xi, wn.repeat(G, 1), wd, G)
    want = d_n_g.double().sum(0, keepdim=True)
    tol = 1e-6 * d_n_g.double().abs().sum(0, keepdim=True) + 1e-30
    assert dns.shape == (1, 6)
    assert bool(((dns.double() - want).abs() <= tol).all()), (dns, want)
    # deterministic
    _, _, dns2, dds2 = run(True)
    assert torch.equal(dns, dns2) and torch.equal(dds, dds2)
    del per_group


def test_modules_take_the_shared_row_path():
    m = kat.KAT_Group(num_groups=8, mode="gelu").cuda()
    x = torch.randn(2, 5, 64, device="cuda", requires_grad=True)
    y = m(x)
    assert type(y.grad_fn).__name__.startswith("KatGroupFunction")
    y.sum().backward()
    assert m.weight_numerator.grad.shape == (1, 6)
    m2 = kat.KAT_Group2D(num_groups=8, mode="identity").cuda()
    y2 = m2(torch.randn(2, 16, 3, 3, device="cuda"))
    assert type(y2.grad_fn).__name__.startswith("KatGroupFunction")


def test_many_groups_take_the_per_group_path():
    """Above SHARED_ROW_MAX_GROUPS groups the modules repeat the numerator (the per-group grid
    reduction is faster there): results and gradients are those of RationalCUDA1DGroup on the
    repeated numerator, bit for bit."""
    from rational_kat_cu_b200.rational_cuda import SHARED_ROW_MAX_GROUPS

    G = 64
    assert G > SHARED_ROW_MAX_GROUPS
    m = kat.KAT_Group(num_groups=G, mode="gelu").cuda()
    g = torch.Generator(device="cpu").manual_seed(9)
    x = torch.randn(16, 768, generator=g).to(torch.bfloat16).cuda().requires_grad_(True)
    gy = torch.randn(16, 768, generator=g).to(torch.bfloat16).cuda()
    y = m(x)
    y.backward(gy)
    xr = x.detach().clone().requires_grad_(True)
    n = m.weight_numerator.detach().clone().requires_grad_(True)
    d = m.weight_denominator.detach().clone().requires_grad_(True)
    yr = RationalCUDA1DGroup.apply(xr, n.repeat(G, 1), d, G)
    yr.backward(gy)
    assert torch.equal(y, yr) and torch.equal(x.grad, xr.grad)
    assert torch.equal(m.weight_numerator.grad, n.grad)
    assert torch.equal(m.weight_denominator.grad, d.grad)
