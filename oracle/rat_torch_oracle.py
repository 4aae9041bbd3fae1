"""ORACLE — test infrastructure only.  Only tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline leg may import this module; the library never does.

A restatement, in PyTorch, of the reference's abs-after-sum activation (the `rat_cuda`
front end of felippe-alves/rational_kat_cu):

  forward       <- the reference's own PyTorch definition, tests/test_correctness.py:16-39
                   (_rat_ref): x viewed [N, G, Dg]; P by Horner from a[5] down to a[0];
                   d by Horner from b[:, 3] down to b[:, 0]; Q = 1 + |x * d|; y = P / Q
                   (the same Horner order as kat_rational/rational_triton.py:56-72)
  backward      <- torch autograd of that forward, except that the sign of D = x d counts
                   as +1 where D == 0, as the reference kernels do
                   (rational_kat_cu/rational_bwd_triton.py:111, where(D < 0, -1, 1));
                   torch's own abs backward would use 0 there
  coefficients  <- rat_cuda's convention (rational_kat_cu/__init__.py:43-46): a [6] shared,
                   expanded to [G, 6] per group; b [G, 4] raw

`compute_dtype=torch.float64` gives the float64 restatement of the same formula.
"""

from __future__ import annotations

import torch


def rat_forward_grouped(x: torch.Tensor, a_grouped: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """y for x [..., D] with per-group numerators a_grouped [G, 6] and denominators b [G, 4]."""
    G = b.shape[0]
    D = x.shape[-1]
    xg = x.reshape(-1, G, D // G)
    num = a_grouped[:, -1].view(1, G, 1)
    for i in range(a_grouped.shape[1] - 2, -1, -1):
        num = a_grouped[:, i].view(1, G, 1) + xg * num
    d = b[:, -1].view(1, G, 1)
    for i in range(b.shape[1] - 2, -1, -1):
        d = b[:, i].view(1, G, 1) + xg * d
    big_d = xg * d
    sign = torch.where(big_d < 0, -1.0, 1.0).to(big_d.dtype).detach()
    den = 1.0 + big_d * sign          # = 1 + |D|, with d|D|/dD = +1 at D = 0
    return (num / den).reshape(x.shape)


def rat_forward_backward(x: torch.Tensor, a: torch.Tensor, b: torch.Tensor,
                         grad_out: torch.Tensor, compute_dtype: torch.dtype = torch.float32,
                         grouped_numerator_grad: bool = False):
    """y, dx, d a, d b as rat_cuda's autograd produces them: d a is [6] (summed over the
    groups), or [G, 6] per group with grouped_numerator_grad=True (what the C ABI returns)."""
    G = b.shape[0]
    xc = x.detach().to(compute_dtype).requires_grad_(True)
    ag = a.detach().to(compute_dtype).reshape(1, -1).expand(G, -1).contiguous().requires_grad_(True)
    bc = b.detach().to(compute_dtype).requires_grad_(True)
    y = rat_forward_grouped(xc, ag, bc)
    y.backward(grad_out.detach().to(compute_dtype))
    da = ag.grad if grouped_numerator_grad else ag.grad.sum(dim=0)
    return y.detach(), xc.grad, da, bc.grad


def rat_magnitudes(x: torch.Tensor, a: torch.Tensor, b: torch.Tensor, grad_out: torch.Tensor):
    """Float64 condition magnitudes for tolerance scaling: per element the absolute-value
    bounds of y and dx (|P|, |D| terms summed in absolute value over |Q|), and per group the
    sums of |terms| of each coefficient gradient ([G, 6] and [G, 4])."""
    G = b.shape[0]
    D = x.shape[-1]
    xg = x.detach().double().reshape(-1, G, D // G)
    go = grad_out.detach().double().reshape(-1, G, D // G)
    ad = a.detach().double().reshape(-1)
    bd = b.detach().double()
    ax = xg.abs()
    pows = [torch.ones_like(ax)]
    for _ in range(5):
        pows.append(pows[-1] * ax)
    pm = sum(ad[k].abs() * pows[k] for k in range(6))
    dpm = sum(k * ad[k].abs() * pows[k - 1] for k in range(1, 6))
    dm = sum(bd[:, j].abs().view(1, G, 1) * pows[j + 1] for j in range(4))
    ddm = sum((j + 1) * bd[:, j].abs().view(1, G, 1) * pows[j] for j in range(4))
    pv = sum(ad[k] * xg ** k for k in range(6))
    dv = sum(bd[:, j].view(1, G, 1) * xg ** (j + 1) for j in range(4))
    q = 1.0 + dv.abs()
    y = pv / q
    y_mag = (pm + y.abs() * dm) / q
    dx_mag = go.abs() * (dpm + y.abs() * ddm + y_mag * ddm) / q
    u = (go / q).abs()
    w = (go * pv / q ** 2).abs()
    w_mag = (go.abs() * y_mag / q)
    num_mag = torch.stack([(u * pows[k]).sum(dim=(0, 2)) for k in range(6)], dim=1)
    den_mag = torch.stack([((w + w_mag) * pows[j + 1]).sum(dim=(0, 2)) for j in range(4)], dim=1)
    return (y_mag.reshape(x.shape), dx_mag.reshape(x.shape), num_mag, den_mag)
