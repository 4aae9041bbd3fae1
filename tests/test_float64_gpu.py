"""float64 tensors: the float64 forward kernel (kat_rational_fwd_f64) for both formulas against
the float64 oracles, and torch.autograd.gradcheck through the KAT autograd Function (float64
forward, fp32 backward — the precisions the reference's kernels use for float64 inputs)."""

import pytest
import torch

import rational_kat_cu_b200 as kat
from oracle import kat_torch_oracle, rat_torch_oracle

pytestmark = pytest.mark.gpu


def test_kat_formula_float64_forward(cuda_device):
    g = torch.Generator().manual_seed(2)
    x = torch.randn(6, 11, 64, generator=g, dtype=torch.float64) * 1.5
    mod = kat.KAT_Group(num_groups=8, mode="gelu").to(cuda_device)
    y = mod(x.to(cuda_device)).cpu()
    assert y.dtype == torch.float64
    ref = kat_torch_oracle.forward(x, mod.weight_numerator.detach().cpu(),
                                   mod.weight_denominator.detach().cpu(), 8,
                                   compute_dtype=torch.float64)
    torch.testing.assert_close(y, ref, rtol=1e-12, atol=1e-12)


def test_kat_formula_float64_nchw_forward(cuda_device):
    g = torch.Generator().manual_seed(3)
    x = torch.randn(2, 16, 5, 5, generator=g, dtype=torch.float64)
    mod = kat.KAT_Group2D(num_groups=4, mode="gelu").to(cuda_device)
    y = mod(x.to(cuda_device)).cpu()
    ref = kat_torch_oracle.forward(x, mod.weight_numerator.detach().cpu(),
                                   mod.weight_denominator.detach().cpu(), 4, layout="nchw",
                                   compute_dtype=torch.float64)
    torch.testing.assert_close(y, ref, rtol=1e-12, atol=1e-12)


def test_abs_sum_formula_float64_forward(cuda_device):
    g = torch.Generator().manual_seed(4)
    x = torch.randn(33, 96, generator=g, dtype=torch.float64) * 2.0
    a = torch.randn(6, generator=g, dtype=torch.float64)
    b = torch.randn(8, 4, generator=g, dtype=torch.float64)
    y = kat.rat_cuda(x.to(cuda_device), a.to(cuda_device), b.to(cuda_device)).cpu()
    ref = rat_torch_oracle.rat_forward_grouped(x, a.view(1, 6).expand(8, 6), b)
    torch.testing.assert_close(y, ref, rtol=1e-12, atol=1e-12)


def test_kat_function_gradcheck(cuda_device):
    g = torch.Generator().manual_seed(5)
    x = (torch.rand(4, 3, 32, generator=g, dtype=torch.float64) * 2 - 1).to(cuda_device)
    mod = kat.KAT_Group(num_groups=4, mode="gelu")
    n = mod.weight_numerator.detach().double().repeat(4, 1).to(cuda_device)
    d = (mod.weight_denominator.detach().double() +
         0.05 * torch.randn(4, 4, generator=g, dtype=torch.float64)).to(cuda_device)
    x.requires_grad_(True)
    n.requires_grad_(True)
    d.requires_grad_(True)
    fn = lambda x, n, d: kat.RationalTriton1DGroup.apply(x, n, d, 4)
    assert torch.autograd.gradcheck(fn, (x, n, d), eps=1e-4, atol=1e-3, rtol=1e-3,
                                    raise_exception=True)
