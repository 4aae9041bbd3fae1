"""Tensor-core GEMMs with the rational activation in the epilogue (include/kat_gemm.h).

  - kat_gemm_bf16 against a float64 product of the same bf16 operands: within half a bf16 ulp
    of the exact value plus the fp32 accumulation bound (K * 2^-23 * sum |a b|), M tails,
    bias on and off;
  - kat_gemm_rational_fwd: h bit-identical to kat_gemm_bf16 (same mainloop and rounding), y
    bit-identical to the activation kernel (KAT_Group's RationalCUDA1DGroup) applied to h;
  - kat_gemm_rational_bwd: dh bit-identical to the activation kernel's backward on
    (h, g = kat_gemm_bf16(a, b)); coefficient gradients within 1e-4 relative of the float64
    oracle on the same (h, g); bit-identical repeats;
  - the KAN block fc1 -> act2 -> fc2 through KANMlpFused against the same block on torch
    linear layers and the activation module, and against a float32 evaluation;
  - the ViT-B/16 MLP size (M = 128 x 197, N = 3072, K = 768, G = 8);
  - the abs-after-sum (rat_cuda) formula through the same kernels."""

import pytest
import torch

import rational_kat_cu_b200 as kat
from oracle import c_oracle
from rational_kat_cu_b200 import _native
from rational_kat_cu_b200 import fused_gemm as fg
from tolerances import assert_coef_grads

pytestmark = pytest.mark.gpu


def _bf16(shape, gen, scale=1.0, device="cuda"):
    return (torch.randn(*shape, generator=gen, device=device) * scale).to(torch.bfloat16)


def _coefs(groups, gen, device="cuda"):
    mod = kat.KAT_Group(num_groups=groups, mode="gelu")
    n = mod.weight_numerator.detach().to(device)
    d = mod.weight_denominator.detach().to(device)
    n = n + 0.01 * torch.randn(n.shape, generator=gen, device=device)
    d = d + 0.01 * torch.randn(d.shape, generator=gen, device=device)
    return n.repeat(groups, 1).contiguous(), d.contiguous()


def _gemm_bound(a, b, bias):
    a64, b64 = a.double(), b.double()
    ref = a64 @ b64.t()
    if bias is not None:
        ref = ref + bias.double()
    mag = a64.abs() @ b64.abs().t()
    k = a.shape[1]
    # bf16 rounding of the result (half an ulp; 2^-8 relative covers it) + fp32 accumulation
    tol = ref.abs() * 2.0 ** -8 + (k + 2) * 2.0 ** -23 * mag + 1e-30
    return ref, tol


SHAPES = [(128, 256, 64), (1, 256, 64), (127, 512, 128), (129, 256, 192), (1000, 768, 256),
          (300, 3072, 768)]


@pytest.mark.parametrize("m,n,k", SHAPES)
@pytest.mark.parametrize("with_bias", [False, True])
def test_gemm_bf16(m, n, k, with_bias):
    gen = torch.Generator(device="cuda").manual_seed(m * 7 + n + k)
    a = _bf16((m, k), gen)
    b = _bf16((n, k), gen, 0.1)
    bias = _bf16((n,), gen) if with_bias else None
    c = fg.gemm_bf16(a, b, bias)
    torch.cuda.synchronize()
    ref, tol = _gemm_bound(a, b, bias)
    err = (c.double() - ref).abs()
    assert bool((err <= tol).all()), f"max err/tol {float((err / tol).max()):.3g}"
    assert fg.device_status(0) == 0


def _fwd_case(m, n, k, groups, seed, with_bias=True):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    a = _bf16((m, k), gen)
    b = _bf16((n, k), gen, k ** -0.5)
    bias = _bf16((n,), gen, 0.1) if with_bias else None
    num, den = _coefs(groups, gen)
    return a, b, bias, num, den


@pytest.mark.parametrize("m,n,k,groups", [(128, 256, 64, 1), (200, 512, 128, 8),
                                          (1000, 768, 256, 8), (333, 3072, 768, 8),
                                          (129, 1024, 64, 32)])
def test_fused_forward_bit_exact(m, n, k, groups):
    a, b, bias, num, den = _fwd_case(m, n, k, groups, seed=m + n)
    h, y = fg.gemm_rational_fwd(a, b, bias, num, den, groups)
    c = fg.gemm_bf16(a, b, bias)
    y_ref = kat.RationalCUDA1DGroup.apply(h, num, den, groups)
    torch.cuda.synchronize()
    assert torch.equal(h, c)
    assert torch.equal(y, y_ref)
    ref, tol = _gemm_bound(a, b, bias)
    assert bool(((h.double() - ref).abs() <= tol).all())


def _bwd_case(m, n, k, groups, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    a = _bf16((m, k), gen)                      # dL/d(fc2 output)
    b = _bf16((n, k), gen, k ** -0.5)           # fc2.weight^T  [hidden, out]
    h = _bf16((m, n), gen, 1.5)                 # pre-activation
    num, den = _coefs(groups, gen)
    return a, b, h, num, den


@pytest.mark.parametrize("m,n,k,groups", [(128, 256, 64, 1), (200, 512, 128, 8),
                                          (1000, 768, 256, 8), (333, 3072, 768, 8),
                                          (129, 1024, 64, 32)])
def test_fused_backward(m, n, k, groups):
    a, b, h, num, den = _bwd_case(m, n, k, groups, seed=3 * m + n)
    dh, d_num, d_den = fg.gemm_rational_bwd(a, b, h, num, den, groups)
    g = fg.gemm_bf16(a, b)
    x_ref = h.detach().clone().requires_grad_(True)
    n_ref = num.detach().clone().requires_grad_(True)
    d_ref = den.detach().clone().requires_grad_(True)
    kat.RationalCUDA1DGroup.apply(x_ref, n_ref, d_ref, groups).backward(g)
    torch.cuda.synchronize()
    assert torch.equal(dh, x_ref.grad)
    o = c_oracle.backward(h.float().reshape(-1).cpu().numpy(), g.float().reshape(-1).cpu().numpy(),
                          num.cpu().numpy(), den.cpu().numpy(), (m, n, 1), groups, want_dx=False)
    assert_coef_grads(d_num.cpu(), o["d_num"], o["d_num_mag"], "d_num")
    assert_coef_grads(d_den.cpu(), o["d_den"], o["d_den_mag"], "d_den")
    # repeats are bit-identical
    dh2, d_num2, d_den2 = fg.gemm_rational_bwd(a, b, h, num, den, groups)
    assert torch.equal(dh, dh2) and torch.equal(d_num, d_num2) and torch.equal(d_den, d_den2)
    assert fg.device_status(0) == 0


def _kan_block(c, hdim, groups, seed):
    torch.manual_seed(seed)
    fc1 = torch.nn.Linear(c, hdim).cuda().to(torch.bfloat16)
    act2 = kat.KAT_Group(num_groups=groups, mode="gelu").cuda()
    fc2 = torch.nn.Linear(hdim, c).cuda().to(torch.bfloat16)
    with torch.no_grad():
        act2.weight_numerator.add_(0.01 * torch.randn_like(act2.weight_numerator))
        act2.weight_denominator.add_(0.01 * torch.randn_like(act2.weight_denominator))
    return fc1, act2, fc2


def _grads(mods):
    return [p.grad.detach().clone() for m in mods for p in m.parameters()]


def test_kan_block_matches_unfused():
    m, c, hdim, groups = 2 * 197, 768, 3072, 8
    fc1, act2, fc2 = _kan_block(c, hdim, groups, seed=5)
    gen = torch.Generator(device="cuda").manual_seed(9)
    x = _bf16((m, c), gen)
    gy = _bf16((m, c), gen, 0.1)

    xf = x.clone().requires_grad_(True)
    out_f = fg.kan_mlp_fused(xf, fc1, act2, fc2)
    out_f.backward(gy)
    grads_f = _grads((fc1, act2, fc2))
    for mod in (fc1, act2, fc2):
        mod.zero_grad(set_to_none=True)

    xu = x.clone().requires_grad_(True)
    out_u = fc2(act2(fc1(xu)))
    out_u.backward(gy)
    grads_u = _grads((fc1, act2, fc2))

    # float32 evaluation of the same block (bf16 parameters upcast)
    x32 = x.float().requires_grad_(True)
    p32 = [p.detach().float().requires_grad_(True) for p in
           (fc1.weight, fc1.bias, act2.weight_numerator, act2.weight_denominator, fc2.weight,
            fc2.bias)]
    h32 = torch.nn.functional.linear(x32, p32[0], p32[1])
    y32 = kat.RationalCUDA1DGroup.apply(h32, p32[2].repeat(groups, 1), p32[3], groups)
    out32 = torch.nn.functional.linear(y32, p32[4], p32[5])
    out32.backward(gy.float())
    grads32 = [p.grad for p in p32]
    torch.cuda.synchronize()

    def rel(a, ref):
        a, ref = a.detach().float(), ref.detach().float()
        return float((a - ref).norm() / ref.norm())

    # fused and unfused bf16 blocks are equally close to the float32 block
    assert rel(out_f, out32) < 1e-2 and rel(out_u, out32) < 1e-2
    assert rel(out_f, out_u) < 1e-2
    assert rel(xf.grad, x32.grad) < 2e-2 and rel(xu.grad, x32.grad) < 2e-2
    for i, (gf, gu, g32) in enumerate(zip(grads_f, grads_u, grads32)):
        assert gf.shape == gu.shape == g32.shape
        assert rel(gf, g32) < 3e-2, f"param {i}: fused {rel(gf, g32):.3g}"
        assert rel(gu, g32) < 3e-2, f"param {i}: unfused {rel(gu, g32):.3g}"


def test_vit_b16_mlp_size():
    m, n, k, groups = 128 * 197, 3072, 768, 8
    a, b, bias, num, den = _fwd_case(m, n, k, groups, seed=11)
    h, y = fg.gemm_rational_fwd(a, b, bias, num, den, groups)
    c = fg.gemm_bf16(a, b, bias)
    y_ref = kat.RationalCUDA1DGroup.apply(h, num, den, groups)
    torch.cuda.synchronize()
    assert torch.equal(h, c) and torch.equal(y, y_ref)
    rows = torch.cat([torch.arange(0, 64), torch.arange(m - 64, m)]).cuda()
    ref, tol = _gemm_bound(a[rows], b, bias)
    assert bool(((h[rows].double() - ref).abs() <= tol).all())

    gen = torch.Generator(device="cuda").manual_seed(12)
    gout = _bf16((m, k), gen, 0.05)
    w2t = _bf16((n, k), gen, k ** -0.5)
    dh, d_num, d_den = fg.gemm_rational_bwd(gout, w2t, h, num, den, groups)
    g = fg.gemm_bf16(gout, w2t)
    x_ref = h.detach().clone().requires_grad_(True)
    n_ref = num.detach().clone().requires_grad_(True)
    d_ref = den.detach().clone().requires_grad_(True)
    kat.RationalCUDA1DGroup.apply(x_ref, n_ref, d_ref, groups).backward(g)
    torch.cuda.synchronize()
    assert torch.equal(dh, x_ref.grad)
    # coefficient gradients: float64 torch restatement on the GPU (same formula as the oracle)
    x64 = h.double()
    g64 = g.double()
    gsz = n // groups
    xg = x64.view(m, groups, gsz)
    gg = g64.view(m, groups, gsz)
    n64 = num.double().view(1, groups, 1, 6)
    c64 = den.double().abs()
    pw = torch.stack([xg ** i for i in range(6)], dim=-1)
    p = (pw * n64).sum(-1)
    q = 1.0 + (pw[..., 1:5] * c64.view(1, groups, 1, 4)).sum(-1)
    dn64 = (gg / q).unsqueeze(-1).mul(pw).sum(dim=(0, 2))
    dd64 = -(gg * p / q ** 2).unsqueeze(-1).mul(pw[..., 1:5]).sum(dim=(0, 2)) * torch.sign(
        den.double())
    assert float(((d_num.double() - dn64).abs() / dn64.abs().clamp_min(1e-3)).max()) < 1e-4
    assert float(((d_den.double() - dd64).abs() / dd64.abs().clamp_min(1e-3)).max()) < 1e-4
    assert fg.device_status(0) == 0


def test_errors():
    a = torch.zeros(128, 64, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        fg.gemm_bf16(a, torch.zeros(100, 64, device="cuda", dtype=torch.bfloat16))
    with pytest.raises(TypeError):
        fg.gemm_bf16(a.float(), torch.zeros(256, 64, device="cuda"))
    with pytest.raises(RuntimeError):
        fg.gemm_bf16(a.cpu(), torch.zeros(256, 64, dtype=torch.bfloat16))
    lib = _native.lib()
    # argument errors come back before anything is enqueued
    assert lib.kat_gemm_bf16(a.data_ptr(), a.data_ptr(), None, a.data_ptr(), 128, 100, 64,
                             None) == _native.KAT_ERR_BAD_SHAPE
    num = torch.zeros(8, 6, device="cuda")
    den = torch.zeros(8, 4, device="cuda")
    out = torch.empty(128, 256, device="cuda", dtype=torch.bfloat16)
    b = torch.zeros(256, 64, device="cuda", dtype=torch.bfloat16)
    assert lib.kat_gemm_rational_fwd(a.data_ptr(), b.data_ptr(), None, num.data_ptr(),
                                     den.data_ptr(), out.data_ptr(), out.data_ptr(), 128, 256, 64,
                                     3, 0, None) == _native.KAT_ERR_BAD_GROUPS
    assert lib.kat_gemm_rational_fwd(a.data_ptr(), b.data_ptr(), None, num.data_ptr(),
                                     den.data_ptr(), out.data_ptr(), out.data_ptr(), 128, 256, 64,
                                     8, 7, None) == _native.KAT_ERR_BAD_FORMULA
    assert lib.kat_gemm_rational_bwd(a.data_ptr(), b.data_ptr(), out.data_ptr(), num.data_ptr(),
                                     den.data_ptr(), out.data_ptr(), num.data_ptr(),
                                     den.data_ptr(), None, 0, 128, 256, 64, 8, 0,
                                     None) == _native.KAT_ERR_WORKSPACE


@pytest.mark.parametrize("m,n,k,groups", [(200, 512, 128, 8), (1000, 3072, 256, 8)])
def test_fused_abs_after_sum_formula(m, n, k, groups):
    """The rat_cuda formula (Q = 1 + |sum b_i x^i|) through the same fused kernels: y and dh
    bit-identical to the activation kernels' abs-after-sum path on the same h and g; the
    coefficient gradients within 1e-4 of the float64 restatement of that formula."""
    from oracle import rat_torch_oracle as rat
    from rational_kat_cu_b200.rat_cuda import rat_bwd_cuda, rat_fwd_cuda

    gen = torch.Generator(device="cuda").manual_seed(m + 7 * n)
    a = _bf16((m, k), gen)
    b = _bf16((n, k), gen, k ** -0.5)
    num = (torch.randn(1, 6, generator=gen, device="cuda") * 0.5).repeat(groups, 1).contiguous()
    den = (torch.randn(groups, 4, generator=gen, device="cuda") * 0.5).contiguous()
    f = _native.KAT_FORMULA_ABS_SUM
    h, y = fg.gemm_rational_fwd(a, b, None, num, den, groups, formula=f)
    assert torch.equal(h, fg.gemm_bf16(a, b))
    assert torch.equal(y, rat_fwd_cuda(h, num, den, groups))
    gout = _bf16((m, k), gen, 0.1)
    dh, d_num, d_den = fg.gemm_rational_bwd(gout, b, h, num, den, groups, formula=f)
    g = fg.gemm_bf16(gout, b)
    dx_ref, dn_ref, dd_ref = rat_bwd_cuda(h, num, den, g, groups)
    torch.cuda.synchronize()
    assert torch.equal(dh, dx_ref)
    _, _, da64, db64 = rat.rat_forward_backward(h.float().cpu(), num[0].cpu(), den.cpu(),
                                                g.float().cpu(), compute_dtype=torch.float64,
                                                grouped_numerator_grad=True)
    _, _, nmag, dmag = rat.rat_magnitudes(h.float().cpu(), num[0].cpu(), den.cpu(),
                                          g.float().cpu())
    assert_coef_grads(d_num.cpu(), da64, nmag, "abs-sum d_num")
    assert_coef_grads(d_den.cpu(), db64, dmag, "abs-sum d_den")


PAIR_CHILD = r'''
import sys
sys.path.insert(0, {repo!r})
import torch
import rational_kat_cu_b200 as kat
from rational_kat_cu_b200 import fused_gemm as fg
g = torch.Generator(device="cuda").manual_seed(21)
m, n, k, G = 1000, 768, 256, 8
a = torch.randn(m, k, generator=g, device="cuda").to(torch.bfloat16)
b = (torch.randn(n, k, generator=g, device="cuda") * k ** -0.5).to(torch.bfloat16)
go = (torch.randn(m, k, generator=g, device="cuda") * 0.1).to(torch.bfloat16)
act = kat.KAT_Group(num_groups=G, mode="gelu").cuda()
num = act.weight_numerator.detach().repeat(G, 1).contiguous()
den = act.weight_denominator.detach().contiguous()
h, y = fg.gemm_rational_fwd(a, b, None, num, den, G)
dh, dn, dd = fg.gemm_rational_bwd(go, b, h, num, den, G)
torch.cuda.synchronize()
assert fg.device_status(0) == 0
torch.save({{"h": h.cpu(), "y": y.cpu(), "dh": dh.cpu(), "dn": dn.cpu(), "dd": dd.cpu()}}, {out!r})
'''


def test_cta_pair_and_single_cta_tiles_agree(tmp_path):
    """The same problem with CTA-pair tiles (cta_group::2, the default where they take no more
    waves) and with one CTA per tile (KAT_GEMM_CTA_PAIR=0): both within the GEMM bound of a
    float64 product, and the fused outputs consistent with each one's own h."""
    import os
    import subprocess
    import sys

    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    outs = {}
    for pair in ("1", "0"):
        out = str(tmp_path / f"pair{pair}.pt")
        env = dict(os.environ, KAT_GEMM_CTA_PAIR=pair)
        res = subprocess.run([sys.executable, "-c", PAIR_CHILD.format(repo=repo, out=out)],
                             env=env, capture_output=True, text=True, timeout=600)
        assert res.returncode == 0, res.stdout + res.stderr
        outs[pair] = torch.load(out)
    g = torch.Generator(device="cuda").manual_seed(21)
    m, n, k = 1000, 768, 256
    a = torch.randn(m, k, generator=g, device="cuda").to(torch.bfloat16)
    b = (torch.randn(n, k, generator=g, device="cuda") * k ** -0.5).to(torch.bfloat16)
    ref, tol = _gemm_bound(a.cpu(), b.cpu(), None)
    for pair, o in outs.items():
        assert bool(((o["h"].double() - ref).abs() <= tol).all()), pair
    d = (outs["1"]["dn"].double() - outs["0"]["dn"].double()).abs()
    assert float((d / outs["0"]["dn"].double().abs().clamp_min(1e-3)).max()) < 1e-3


STALL_CHILD = r'''
import os, sys, time
sys.path.insert(0, {repo!r})
import torch
from rational_kat_cu_b200 import _native
from rational_kat_cu_b200 import fused_gemm as fg
a = torch.randn(300, 128, device="cuda").to(torch.bfloat16)
b = (torch.randn(512, 128, device="cuda") * 0.1).to(torch.bfloat16)
assert fg.device_status(0, reset=True) == 0
_native.lib().kat_gemm_set_test_stall(1)
t0 = time.time()
fg.gemm_bf16(a, b)
torch.cuda.synchronize()
waited = time.time() - t0
status = fg.device_status(0, reset=True)
_native.lib().kat_gemm_set_test_stall(0)
c = fg.gemm_bf16(a, b)
torch.cuda.synchronize()
err = float((c.double() - a.double() @ b.double().t()).abs().max())
print("result", status, round(waited, 2), err, fg.device_status(0))
'''


def test_stalled_pipeline_reports_and_recovers():
    """A pipeline wait that nothing completes (test hook kat_gemm_set_test_stall(1): the MMA issuer
    waits on a barrier no one arrives at) runs out after its clock limit: the kernel returns,
    the sticky status reads KAT_DEVICE_WAIT_TIMEOUT, tensor memory is freed, and the next
    launch in the same context computes correctly."""
    import os
    import subprocess
    import sys

    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ)
    res = subprocess.run([sys.executable, "-c", STALL_CHILD.format(repo=repo)], env=env,
                         capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stdout + res.stderr
    line = [l for l in res.stdout.splitlines() if l.startswith("result")][-1].split()
    status, waited, err, after = int(line[1]), float(line[2]), float(line[3]), int(line[4])
    assert status == _native.KAT_DEVICE_WAIT_TIMEOUT
    assert 0.5 < waited < 60.0
    assert err < 0.05 and after == 0


def test_inference_forward_writes_y_only():
    """h = NULL (no backward follows): y identical to the h-storing forward; the KAN block
    under no_grad takes this form and matches the training-mode output."""
    a, b, bias, num, den = _fwd_case(333, 3072, 768, 8, seed=77)
    h, y = fg.gemm_rational_fwd(a, b, bias, num, den, 8)
    none, y2 = fg.gemm_rational_fwd(a, b, bias, num, den, 8, need_h=False)
    torch.cuda.synchronize()
    assert none is None and torch.equal(y, y2)
    fc1, act2, fc2 = _kan_block(768, 3072, 8, seed=3)
    x = _bf16((2 * 197, 768), torch.Generator(device="cuda").manual_seed(4))
    with torch.no_grad():
        out_inf = fg.kan_mlp_fused(x, fc1, act2, fc2)
    out_train = fg.kan_mlp_fused(x.clone().requires_grad_(True), fc1, act2, fc2)
    assert torch.equal(out_inf, out_train.detach())


def test_empty_batch():
    """M = 0: the forward returns empty outputs, the backward empty dh and zero coefficient
    gradients (the sums over no elements), like the activation kernels' empty inputs."""
    a = torch.empty(0, 128, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(512, 128, device="cuda").to(torch.bfloat16)
    num, den = _coefs(8, torch.Generator(device="cuda").manual_seed(1))
    h, y = fg.gemm_rational_fwd(a, b, None, num, den, 8)
    assert h.shape == (0, 512) and y.shape == (0, 512)
    dh, dn, dd = fg.gemm_rational_bwd(a, b, h, num, den, 8)
    torch.cuda.synchronize()
    assert dh.shape == (0, 512)
    assert bool((dn == 0).all()) and bool((dd == 0).all())
    assert fg.gemm_bf16(a, b).shape == (0, 512)
