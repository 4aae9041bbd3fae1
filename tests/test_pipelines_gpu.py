"""Every streaming design of the library gives the same results within the parity rules:
KAT_RATIONAL_PIPELINE = async (default: register-prefetch forward, cp.async-ring backward),
registers (register prefetch for both) and bulk (producer-warp cp.async.bulk ring).  The
mode is read once per process, so each runs in a child process over golden cases and an
odd-shaped NCHW case, and must also leave the device status word clear."""

import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r'''
import sys
sys.path.insert(0, {repo!r}); sys.path.insert(0, {tests!r})
import torch
from golden_data import load_case
from test_parity_gpu import run_module, oracle_for, assert_parity, _random_case, _dims
from golden_data import TORCH_DTYPES
from rational_kat_cu_b200 import _native
dev = torch.device("cuda", 0)
for name in ["gelu_blc_f32", "gelu_pert_blc_bf16", "gelu_blc_f16", "gelu_nchw_f32",
             "g64_blc_bf16", "odd_group_f32"]:
    c = load_case(name)
    out = run_module(c["x"], c["grad_out"], c["w_num"], c["w_den"], c["G"], c["layout"], dev,
                     TORCH_DTYPES[c["dtype"]])
    assert_parity(out, (c["y"], c["dx"]), oracle_for(c["x"], c["grad_out"], c["w_num"],
                  c["w_den"], c["dims"], c["G"]), c["dtype"], name)
for shape, groups, layout, dtype in [((37, 5, 3072), 8, "blc", "bf16"),
                                     ((3, 64, 28, 28), 8, "nchw", "f32"),
                                     ((2, 3, 8192), 64, "blc", "f16")]:
    x, gy, wn, wd = _random_case(shape, groups, layout, dtype)
    out = run_module(x, gy, wn, wd, groups, layout, dev, TORCH_DTYPES[dtype])
    assert_parity(out, None, oracle_for(x, gy, wn, wd, _dims(shape, layout), groups), dtype,
                  str(shape))
assert _native.device_status(0) == 0
print("ok")
'''


@pytest.mark.parametrize("mode", ["async", "registers", "bulk"])
def test_pipeline_mode_parity(mode):
    env = dict(os.environ, KAT_RATIONAL_PIPELINE=mode)
    code = CHILD.format(repo=REPO, tests=os.path.join(REPO, "tests"))
    res = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True,
                         timeout=600)
    assert res.returncode == 0 and res.stdout.strip().endswith("ok"), res.stdout + res.stderr



HASH_CHILD = r'''
import sys, hashlib
sys.path.insert(0, {repo!r})
import torch
import rational_kat_cu_b200 as kat
torch.manual_seed(0)
x = torch.randn(64, 197, 3072, device="cuda").to(torch.bfloat16).requires_grad_(True)
m = kat.KAT_Group(num_groups=8, mode="gelu").cuda()
y = m(x)
y.backward(torch.randn_like(y))
torch.cuda.synchronize()
h = hashlib.sha256()
for t in (y, x.grad, m.weight_numerator.grad, m.weight_denominator.grad):
    h.update(t.detach().float().cpu().numpy().tobytes())
print("hash", h.hexdigest())
'''


def test_grid_reduction_launch_modes_agree():
    """The grid reduction launched as a programmatic dependent of the partial-sum kernel
    (default) and as an ordinary launch (KAT_RATIONAL_PDL=0) give bit-identical results."""
    code = HASH_CHILD.format(repo=REPO)
    hashes = []
    for pdl in ("1", "0"):
        env = dict(os.environ, KAT_RATIONAL_PDL=pdl)
        res = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True,
                             text=True, timeout=600)
        assert res.returncode == 0, res.stdout + res.stderr
        hashes.append([l for l in res.stdout.splitlines() if l.startswith("hash")][-1])
    assert hashes[0] == hashes[1]
