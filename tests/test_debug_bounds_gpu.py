"""The bounds-checked debug build (libkat_rational_debug.so, -DKAT_DEBUG_BOUNDS=1), the GPU-side
stand-in for compute-sanitizer (closed on the GPU pool): every global access, workspace slot and
plan invariant of the activation kernels is checked before it is made, and a violation sets
KAT_DEVICE_BOUNDS in the device status word instead of faulting.

On the edge shapes (odd and 3-wide groups, [B, C], 7x7 NCHW, several column blocks, one
element per group, 257 rows, 12-wide groups on 8-byte vectors, misaligned pointers, empty
input, short and wide problems on 512-column backward tiles, blocks aligned unevenly to
column blocks), for every dtype, both formulas and each streaming design (cp.async ring, register
prefetch, bulk-copy ring), forward and backward through the debug build must leave the status
word at 0 and give results bit-identical to the release build.
"""

import ctypes
import os
import subprocess
import sys

import pytest
import torch

from rational_kat_cu_b200 import _build, _native

pytestmark = pytest.mark.gpu
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CASES = [
    # (batch, channels, inner), groups, dtype, element offset of every tensor
    ((5, 36, 1), 12, "f32", 0),           # 3-wide groups: scalar vectors
    ((7, 36, 1), 12, "bf16", 0),
    ((33, 768, 1), 8, "bf16", 0),         # [B, C]
    ((4, 197 * 2, 1), 2, "f16", 0),
    ((3, 64, 49), 8, "f32", 0),           # 7x7 NCHW: odd inner extent
    ((2, 16, 49), 4, "bf16", 0),
    ((2, 8192, 1), 16, "bf16", 0),        # several column blocks
    ((2, 8192, 1), 64, "f32", 0),
    ((9, 32, 1), 32, "f32", 0),           # one element per group
    ((257, 256, 1), 8, "f16", 0),         # 257 rows
    ((6, 768, 1), 64, "bf16", 0),         # 12-wide groups: 8-byte vectors
    ((11, 768, 1), 8, "bf16", 1),         # misaligned pointers: scalar path
    ((5, 96, 1), 4, "f32", 3),
    ((0, 768, 1), 8, "bf16", 0),          # empty input
    ((128, 3072, 1), 8, "bf16", 0),       # the headline layout, a few rows
    ((4, 64, 3136), 8, "f32", 0),         # short, wide NCHW: 512-column backward tiles
    ((4, 262144, 1), 8, "bf16", 0),       # short, wide [B, C]: 512-column backward tiles
    ((37, 8192, 1), 8, "bf16", 0),        # blocks aligned to 8 column blocks, unevenly
    ((300, 6144, 1), 16, "f16", 0),       # blocks aligned to 6 column blocks, unevenly
]
CODES = {"f32": (torch.float32, _native.KAT_DTYPE_F32), "bf16": (torch.bfloat16, _native.KAT_DTYPE_BF16),
         "f16": (torch.float16, _native.KAT_DTYPE_F16)}


def _debug_lib():
    path = _build.DEBUG_LIBRARY
    if not os.path.exists(path):
        pytest.fail(f"{path} missing: build it with python -m rational_kat_cu_b200._build --debug")
    lib = ctypes.CDLL(path)
    _native._declare(lib)
    return lib


def _status(lib, reset=True):
    out = ctypes.c_int(0)
    assert lib.kat_rational_device_status(0, 1 if reset else 0, ctypes.byref(out)) == 0
    return out.value


def _run(lib, dims, groups, dtype, offset, formula, seed=0):
    tdt, code = CODES[dtype]
    n = dims[0] * dims[1] * dims[2]
    g = torch.Generator(device="cpu").manual_seed(seed)

    def buf(vals):
        t = torch.empty(n + offset + 8, dtype=tdt, device="cuda")
        t[offset:offset + n] = vals.to(tdt)
        return t

    x = buf(torch.randn(n, generator=g) * 1.5)
    gy = buf(torch.randn(n, generator=g))
    y, dx = buf(torch.zeros(n)), buf(torch.zeros(n))
    num = (torch.randn(groups, 6, generator=g) * 0.3).cuda()
    den = (torch.randn(groups, 4, generator=g) * 0.3).cuda()
    dn = torch.empty(groups, 6, device="cuda")
    dd = torch.empty(groups, 4, device="cuda")
    need = ctypes.c_size_t(0)
    _native.check("ws", lib.kat_rational_bwd_workspace_size(*dims, groups, code, 0,
                                                            ctypes.byref(need)))
    ws = torch.empty(max(need.value, 16), dtype=torch.uint8, device="cuda")
    ptr = lambda t: t.data_ptr() + offset * t.element_size()  # noqa: E731
    sp = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _native.check("fwd", lib.kat_rational_fwd_formula(ptr(x), ptr(y), num.data_ptr(),
                                                      den.data_ptr(), *dims, groups, code,
                                                      formula, sp))
    _native.check("bwd", lib.kat_rational_bwd_formula(
        ptr(x), ptr(gy), ptr(dx), num.data_ptr(), den.data_ptr(), dn.data_ptr(), dd.data_ptr(),
        ws.data_ptr(), ws.numel(), *dims, groups, code, formula, sp))
    torch.cuda.synchronize()
    return y[offset:offset + n].clone(), dx[offset:offset + n].clone(), dn.clone(), dd.clone()


def _same(a, b):
    return torch.equal(a.view(torch.int16 if a.element_size() == 2 else torch.int32),
                       b.view(torch.int16 if b.element_size() == 2 else torch.int32))


@pytest.mark.parametrize("formula", [_native.KAT_FORMULA_KAT, _native.KAT_FORMULA_ABS_SUM])
@pytest.mark.parametrize("dims,groups,dtype,offset", CASES)
def test_debug_build_clean_and_identical(dims, groups, dtype, offset, formula):
    dbg = _debug_lib()
    rel = _native.lib()
    _status(dbg)
    got = _run(dbg, dims, groups, dtype, offset, formula)
    assert _status(dbg) == 0, "a bounds check failed in the debug build"
    want = _run(rel, dims, groups, dtype, offset, formula)
    for g_, w_, name in zip(got, want, ("y", "dx", "d_num", "d_den")):
        assert _same(g_, w_), f"{name} differs between the debug and release builds"


CHILD = r'''
import sys
sys.path.insert(0, {repo!r})
sys.path.insert(0, {tests!r})
import test_debug_bounds_gpu as t
from rational_kat_cu_b200 import _native
dbg = t._debug_lib()
rel = _native.lib()
bad = 0
for dims, groups, dtype, offset in t.CASES:
    t._status(dbg)
    got = t._run(dbg, dims, groups, dtype, offset, _native.KAT_FORMULA_KAT)
    st = t._status(dbg)
    want = t._run(rel, dims, groups, dtype, offset, _native.KAT_FORMULA_KAT)
    same = all(t._same(a, b) for a, b in zip(got, want))
    if st != 0 or not same:
        bad += 1
        print("FAIL", dims, groups, dtype, offset, st, same)
print("done", bad)
'''


@pytest.mark.parametrize("pipeline", ["registers", "bulk"])
def test_debug_build_other_streaming_designs(pipeline):
    """The register-prefetch and bulk-copy designs (selected once per process by
    KAT_RATIONAL_PIPELINE) through the debug build, in a child process."""
    env = dict(os.environ, KAT_RATIONAL_PIPELINE=pipeline)
    code = CHILD.format(repo=REPO, tests=os.path.join(REPO, "tests"))
    res = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True,
                         timeout=600, cwd=REPO)
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-3000:]
    assert "done 0" in res.stdout, res.stdout[-3000:]
