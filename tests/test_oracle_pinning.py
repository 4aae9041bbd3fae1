"""The oracle is pinned to the reference before it is trusted (CPU only).

Golden vectors come from running the reference's own PyTorch implementation
(tests/golden/make_golden.py).  Checks:
  - the torch restatement (oracle/kat_torch_oracle.py) reproduces them, bit for bit on
    the forward and input gradient (same op sequence), to fp32 reduction noise on the
    coefficient gradients;
  - the float64 C restatement (oracle/kat_oracle.c) agrees with them within the fp32
    rounding of the reference (condition-aware);
  - the known answers: 'identity' coefficients give y == x and d_denominator == 0.
"""

import numpy as np
import pytest
import torch

from golden_data import case_names, load_case, load_cfg1
from oracle import c_oracle
from oracle import kat_torch_oracle as torch_oracle
from tolerances import assert_coef_grads, assert_elementwise


def _c_oracle_case(c):
    G = c["G"]
    x = c["x"].reshape(-1).numpy()
    y, ymag = c_oracle.forward(x, c["w_num"].numpy(), c["w_den"].numpy(), c["dims"], G)
    b = c_oracle.backward(x, c["grad_out"].reshape(-1).numpy(), c["w_num"].numpy(),
                          c["w_den"].numpy(), c["dims"], G)
    return y, ymag, b


@pytest.mark.parametrize("name", case_names())
def test_torch_restatement_reproduces_reference(name):
    c = load_case(name)
    y, dx, dn, dd = torch_oracle.forward_backward(c["x"], c["w_num"], c["w_den"], c["G"],
                                                  c["grad_out"], layout=c["layout"])
    assert torch.equal(y, c["y"]), name
    assert torch.equal(dx, c["dx"]), name
    torch.testing.assert_close(dn, c["d_num"], rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(dd, c["d_den"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("name", case_names())
def test_c_oracle_agrees_with_reference(name):
    c = load_case(name)
    y, ymag, b = _c_oracle_case(c)
    assert_elementwise(c["y"], y, ymag, "f32", f"{name}/y")
    assert_elementwise(c["dx"], b["dx"], b["dx_mag"], "f32", f"{name}/dx")
    # The reference's fp32 coefficient gradients against the float64 restatement.
    assert_coef_grads(c["d_num"], b["d_num"].sum(0, keepdims=True),
                      b["d_num_mag"].sum(0, keepdims=True), f"{name}/d_num")
    assert_coef_grads(c["d_den"], b["d_den"], b["d_den_mag"], f"{name}/d_den")


@pytest.mark.parametrize("name", ["identity_blc_f32", "identity_nchw_f32", "mode_identity"])
def test_identity_known_answer(name):
    c = load_case(name)
    assert torch.equal(c["y"], c["x"])
    assert torch.equal(c["dx"], c["grad_out"])
    assert torch.count_nonzero(c["d_den"]) == 0
    y, _, b = _c_oracle_case(c)
    assert np.array_equal(y, c["x"].reshape(-1).numpy().astype(np.float64))
    assert np.count_nonzero(b["d_den"]) == 0


def test_gelu_preset_is_reference_table():
    """init.json ships unchanged: the 'gelu' row the golden cases used."""
    from rational_kat_cu_b200._init_table import load_table

    c = load_case("gelu_blc_f32")
    t = load_table()["gelu"]
    assert np.array_equal(c["w_num"].numpy().ravel(),
                          np.asarray(t["init_w_numerator"], np.float32))
    assert np.array_equal(c["w_den"].numpy()[0], np.asarray(t["init_w_denominator"], np.float32))


def test_cfg1_workload_and_oracles():
    """x[8,197,768] fp32, G=8, 'gelu': regenerated inputs match the golden checksums, the
    torch restatement reproduces the reference's sampled outputs and gradients, and the
    float64 oracle agrees with them."""
    from rational_kat_cu_b200.workloads import kat_group_f32

    g = load_cfg1()
    w = kat_group_f32()
    x, gy = w.inputs()
    assert tuple(g["shape"]) == w.shape
    assert float(x.double().sum()) == pytest.approx(float(g["x_sum"]), rel=0, abs=1e-9)
    assert float((x.double() ** 2).sum()) == pytest.approx(float(g["x_sumsq"]), rel=1e-12)
    idx = g["index"]
    assert np.array_equal(x.reshape(-1).numpy()[idx], g["x_sample"])
    wn, wd = w.coefficients()
    assert np.array_equal(wn.numpy(), g["w_num"]) and np.array_equal(wd.numpy(), g["w_den"])

    y, dx, dn, dd = torch_oracle.forward_backward(x, wn, wd, w.groups, gy)
    assert np.array_equal(y.reshape(-1).numpy()[idx], g["y_sample"])
    assert np.array_equal(dx.reshape(-1).numpy()[idx], g["dx_sample"])
    np.testing.assert_allclose(dn.numpy(), g["d_num"], rtol=1e-4)
    np.testing.assert_allclose(dd.numpy(), g["d_den"], rtol=1e-4)

    y64, ymag = c_oracle.forward(x.reshape(-1).numpy(), wn.numpy(), wd.numpy(), w.dims(),
                                 w.groups)
    b = c_oracle.backward(x.reshape(-1).numpy(), gy.reshape(-1).numpy(), wn.numpy(),
                          wd.numpy(), w.dims(), w.groups)
    assert_elementwise(g["y_sample"], y64[idx], ymag[idx], "f32", "cfg1/y")
    assert_elementwise(g["dx_sample"], b["dx"][idx], b["dx_mag"][idx], "f32", "cfg1/dx")
    assert_coef_grads(g["d_num"], b["d_num"].sum(0, keepdims=True),
                      b["d_num_mag"].sum(0, keepdims=True), "cfg1/d_num")
    assert_coef_grads(g["d_den"], b["d_den"], b["d_den_mag"], "cfg1/d_den")


def test_planted_oracle_mistake_is_caught():
    """A wrong formula in the oracle (abs applied after the sum, as the reference's Triton
    kernels do) must fail the parity rule on the golden data."""
    c = load_case("random_blc_f32")
    G = c["G"]
    x = c["x"].reshape(-1, c["shape"][-1])
    wn = c["w_num"].repeat(G, 1)
    per = c["shape"][-1] // G
    g_idx = torch.arange(c["shape"][-1]) // per
    a = wn[g_idx].T            # [6, C]
    b = c["w_den"][g_idx].T    # [4, C]
    p = sum(a[k] * x ** k for k in range(6))
    q = 1 + (sum(b[i] * x ** (i + 1) for i in range(4))).abs()
    wrong = (p / q).reshape(-1).numpy()
    _, ymag, _ = _c_oracle_case(c)
    with pytest.raises(AssertionError):
        assert_elementwise(wrong, c["y"].reshape(-1).numpy(), ymag, "f32", "planted")
