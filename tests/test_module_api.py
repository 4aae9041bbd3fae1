"""Drop-in API of the modules and Functions (CPU): constructor, presets, parameter names
and shapes, state_dict compatibility, export names, argument checks, and the explicit
device='cpu' formulation against the oracle."""

import numpy as np
import pytest
import torch

import kat_rational
import rational_kat_cu_b200 as kat
from oracle import c_oracle
from oracle import kat_torch_oracle as torch_oracle
from rational_kat_cu_b200._init_table import load_table
from tolerances import assert_coef_grads, assert_elementwise


def test_reference_export_names():
    for name in ("KAT_Group", "KAT_Group2D", "KAT_Group_Torch", "RationalTriton1DGroup"):
        assert hasattr(kat_rational, name)
    assert kat.RationalTriton1DGroup is kat.RationalCUDA1DGroup
    assert kat.RationalTriton2D is kat.RationalCUDA2D
    assert kat_rational.KAT_Group is kat.KAT_Group


@pytest.mark.parametrize("cls", [kat.KAT_Group, kat.KAT_Group2D, kat.KAT_Group_Torch])
def test_parameters_and_state_dict(cls):
    m = cls(num_groups=8, mode="gelu") if cls is kat.KAT_Group_Torch else cls()
    sd = m.state_dict()
    assert list(sd) == ["weight_numerator", "weight_denominator"]
    assert sd["weight_numerator"].shape == (1, 6) and sd["weight_numerator"].dtype == torch.float32
    assert sd["weight_denominator"].shape == (8, 4)
    table = load_table()["gelu"]
    assert np.allclose(sd["weight_numerator"].numpy()[0], table["init_w_numerator"])
    assert np.allclose(sd["weight_denominator"].numpy(), [table["init_w_denominator"]] * 8)
    assert m.order == (5, 4)
    assert "num_groups=8" in m.extra_repr()


def test_state_dict_interchange():
    a = kat.KAT_Group(num_groups=4, mode="swish")
    b = kat.KAT_Group2D(num_groups=4, mode="gelu")
    c = kat.KAT_Group_Torch(num_groups=4, mode="tanh")
    b.load_state_dict(a.state_dict())
    c.load_state_dict(a.state_dict())
    assert torch.equal(b.weight_denominator, a.weight_denominator)
    assert torch.equal(c.weight_numerator, a.weight_numerator)


@pytest.mark.parametrize("mode", list(load_table()))
def test_every_preset_loads(mode):
    m = kat.KAT_Group(num_groups=2, mode=mode)
    t = load_table()[mode]
    assert np.allclose(m.weight_numerator.detach().numpy()[0], t["init_w_numerator"])
    assert np.allclose(m.weight_denominator.detach().numpy()[1], t["init_w_denominator"])


def test_unknown_preset_raises_keyerror():
    with pytest.raises(KeyError):
        kat.KAT_Group(mode="no_such_mode")


def test_device_argument_checks():
    with pytest.raises(AssertionError):
        kat.KAT_Group(device="tpu")
    with pytest.raises(AssertionError, match="Only CUDA"):
        kat.KAT_Group2D(device="cpu")


def test_cuda_module_refuses_cpu_tensors():
    m = kat.KAT_Group()
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        m(torch.randn(2, 3, 16))
    m2 = kat.KAT_Group2D()
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        m2(torch.randn(2, 16, 3, 3))


def test_input_rank_checks():
    with pytest.raises(AssertionError):
        kat.KAT_Group(device="cpu")(torch.randn(2, 3, 4, 16))
    with pytest.raises(AssertionError):
        kat.KAT_Group2D()(torch.randn(2, 16))


def test_function_checks_coefficient_counts():
    x = torch.randn(2, 16)
    with pytest.raises(AssertionError, match="numerator"):
        kat.rational_fwd_cuda(x, torch.zeros(3, 6), torch.zeros(4, 4), 4)


@pytest.mark.parametrize("shape,groups", [((2, 5, 64), 8), ((6, 48), 4), ((3, 4, 36), 12)])
def test_cpu_formulation_matches_oracle(shape, groups):
    """device='cpu' performs the reference's sequence of tensor operations: y and every
    gradient equal the oracle's restatement of that sequence bit for bit (and are within
    the condition-aware bounds of float64)."""
    m = kat.KAT_Group(num_groups=groups, mode="gelu", device="cpu")
    with torch.no_grad():
        m.weight_denominator.add_(torch.randn(groups, 4,
                                              generator=torch.Generator().manual_seed(5)) * 0.05)
    x = torch.randn(*shape, generator=torch.Generator().manual_seed(0)).requires_grad_(True)
    gy = torch.randn(*shape, generator=torch.Generator().manual_seed(1))
    y = m(x)
    y.backward(gy)
    dims = (x.numel() // shape[-1], shape[-1], 1)
    wn, wd = m.weight_numerator.detach(), m.weight_denominator.detach()
    y64, ymag = c_oracle.forward(x.detach().reshape(-1).numpy(), wn.numpy(), wd.numpy(), dims,
                                 groups)
    b = c_oracle.backward(x.detach().reshape(-1).numpy(), gy.reshape(-1).numpy(), wn.numpy(),
                          wd.numpy(), dims, groups)
    assert_elementwise(y, y64, ymag, "f32", "cpu/y")
    assert_elementwise(x.grad, b["dx"], b["dx_mag"], "f32", "cpu/dx")
    assert_coef_grads(m.weight_numerator.grad, b["d_num"].sum(0), b["d_num_mag"].sum(0),
                      "cpu/d_num")
    assert_coef_grads(m.weight_denominator.grad, b["d_den"], b["d_den_mag"], "cpu/d_den")
    # and equals the reference op sequence (oracle restatement) bit for bit
    layout = "blc" if len(shape) == 3 else "bc"
    ry, rdx, rdn, rdd = torch_oracle.forward_backward(x.detach(), wn, wd, groups, gy,
                                                      layout=layout)
    assert torch.equal(y.detach(), ry)
    assert torch.equal(x.grad, rdx)
    assert torch.equal(m.weight_numerator.grad, rdn)
    assert torch.equal(m.weight_denominator.grad, rdd)


def test_torch_module_matches_cpu_kat_group():
    x = torch.randn(2, 3, 32)
    a = kat.KAT_Group_Torch(num_groups=4, mode="gelu")(x)
    b = kat.KAT_Group(num_groups=4, mode="gelu", device="cpu")(x)
    assert torch.equal(a, b)
