"""HostPipeline (host-buffer forward+backward with overlapped copies) gives the same y and
dx as one device-resident call, bit for bit (elementwise results do not depend on the
chunking), and coefficient gradients within the 1e-4 bar of the float64 oracle."""

import pytest
import torch

import rational_kat_cu_b200 as kat
from oracle import c_oracle
from rational_kat_cu_b200.host_io import HostPipeline
from tolerances import assert_coef_grads

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape,groups,dtype,layout,chunks", [
    ((24, 197, 768), 8, torch.bfloat16, "blc", 5),
    ((7, 3, 256), 4, torch.float32, "blc", 16),
    ((6, 64, 14, 14), 8, torch.float32, "nchw", 3),
])
def test_host_pipeline_matches_device_call(shape, groups, dtype, layout, chunks):
    dev = torch.device("cuda", 0)
    gen = torch.Generator().manual_seed(5)
    x = torch.randn(*shape, generator=gen).to(dtype)
    gy = torch.randn(*shape, generator=gen).to(dtype)
    cls = kat.KAT_Group2D if layout == "nchw" else kat.KAT_Group
    mod = cls(num_groups=groups, mode="gelu").to(dev)
    with torch.no_grad():
        mod.weight_denominator.add_(0.01 * torch.randn(groups, 4, generator=gen).to(dev))
    xd = x.to(dev).requires_grad_(True)
    y_ref = mod(xd)
    y_ref.backward(gy.to(dev))
    ref_num = mod.weight_numerator.grad.clone()
    ref_den = mod.weight_denominator.grad.clone()

    h_x, h_gy = x.pin_memory(), gy.pin_memory()
    h_y = torch.empty_like(h_x).pin_memory()
    h_dx = torch.empty_like(h_x).pin_memory()
    h_grads = [torch.empty(1, 6).pin_memory(), torch.empty(groups, 4).pin_memory()]
    pipe = HostPipeline(mod, chunks=chunks)
    for call in range(3):   # later calls reuse the device buffers; the last one overlaps
        mod.zero_grad(set_to_none=True)
        pipe.run(h_x, h_gy, h_y, h_dx, grads_host=h_grads, wait=call < 2)
        pipe.wait()
        torch.cuda.synchronize()
        assert torch.equal(h_y, y_ref.detach().cpu())
        assert torch.equal(h_dx, xd.grad.cpu())
        torch.testing.assert_close(h_grads[0], ref_num.cpu(), rtol=1e-4, atol=1e-4)
        torch.testing.assert_close(h_grads[1], ref_den.cpu(), rtol=1e-4, atol=1e-4)
    if layout == "nchw":
        dims = (shape[0], shape[1], shape[2] * shape[3])
    else:
        dims = (x.numel() // shape[-1], shape[-1], 1)
    b = c_oracle.backward(x.float().reshape(-1).numpy(), gy.float().reshape(-1).numpy(),
                          mod.weight_numerator.detach().cpu().numpy(),
                          mod.weight_denominator.detach().cpu().numpy(), dims, groups,
                          want_dx=False)
    assert_coef_grads(h_grads[0], b["d_num"].sum(0, keepdims=True),
                      b["d_num_mag"].sum(0, keepdims=True), "pipeline d_num")
    assert_coef_grads(h_grads[1], b["d_den"], b["d_den_mag"], "pipeline d_den")


def test_host_pipeline_abs_sum_formula():
    """A RatGroup (rat_cuda's abs-after-sum formula) through the pipeline gives the same y
    and dx as the device-resident rat_cuda call, and its coefficient gradients (numerator
    [6], denominator [G, 4]) within 1e-4 of the float64 oracle."""
    from oracle import rat_torch_oracle as rat

    dev = torch.device("cuda", 0)
    gen = torch.Generator().manual_seed(8)
    G = 8
    x = torch.randn(40, 197, 768, generator=gen).to(torch.bfloat16)
    gy = torch.randn(40, 197, 768, generator=gen).to(torch.bfloat16)
    a = torch.randn(6, generator=gen) * 0.5
    b = torch.randn(G, 4, generator=gen) * 0.5
    mod = kat.RatGroup(num_groups=G, numerator=a, denominator=b).to(dev)
    xd = x.to(dev).requires_grad_(True)
    y_ref = mod(xd)
    y_ref.backward(gy.to(dev))
    h_x, h_gy = x.pin_memory(), gy.pin_memory()
    h_y = torch.empty_like(h_x).pin_memory()
    h_dx = torch.empty_like(h_x).pin_memory()
    h_grads = [torch.empty(6).pin_memory(), torch.empty(G, 4).pin_memory()]
    ref_num = mod.weight_numerator.grad.clone()
    mod.zero_grad(set_to_none=True)
    pipe = HostPipeline(mod, chunks=6)
    pipe.run(h_x, h_gy, h_y, h_dx, grads_host=h_grads)
    torch.cuda.synchronize()
    assert torch.equal(h_y, y_ref.detach().cpu())
    assert torch.equal(h_dx, xd.grad.cpu())
    torch.testing.assert_close(h_grads[0], ref_num.cpu(), rtol=1e-4, atol=1e-4)
    _, _, da64, db64 = rat.rat_forward_backward(x.float().reshape(-1, 768), a, b,
                                                gy.float().reshape(-1, 768),
                                                compute_dtype=torch.float64)
    _, _, nmag, dmag = rat.rat_magnitudes(x.float().reshape(-1, 768), a, b,
                                          gy.float().reshape(-1, 768))
    assert_coef_grads(h_grads[0], da64, nmag.sum(0), "pipeline rat d_num")
    assert_coef_grads(h_grads[1], db64, dmag, "pipeline rat d_den")
