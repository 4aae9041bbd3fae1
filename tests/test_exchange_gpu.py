"""The data-parallel backward (kat_rational_bwd_allreduce): the coefficient-gradient
exchange fused into the reduction kernel over NVLink peer memory.

  - world size 1 reproduces kat_rational_bwd bit for bit;
  - a wait that runs out (a second rank that never arrives: both "ranks" point at one
    buffer, so nothing ever raises rank 1's flag) sets KAT_DEVICE_EXCHANGE_TIMEOUT, writes
    NaN gradients, leaves dx intact and the context usable;
  - a word tagged with a call out of step is refused at once (NaN, status, broken buffer),
    and a broken buffer fails the next call at once without posting anything;
  - with two GPUs, two processes get identical gradients equal to the rank-order average of
    their local gradients, then tear the buffers down collectively (skipped on one-GPU
    machines).
"""

import ctypes
import os
import socket
import subprocess
import sys
import tempfile

import pytest
import torch

from rational_kat_cu_b200 import _native

pytestmark = pytest.mark.gpu
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _problem(dev, rows=4 * 197, C=768, G=8, dtype=torch.bfloat16, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, C, generator=g).to(dtype).to(dev)
    gy = torch.randn(rows, C, generator=g).to(dtype).to(dev)
    n = (torch.randn(G, 6, generator=g) * 0.3).to(dev)
    d = (torch.randn(G, 4, generator=g) * 0.3).to(dev)
    return x, gy, n, d


def _call(lib_fn, x, gy, n, d, G, peers=None):
    dev = x.device
    code = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}[x.dtype]
    rows, C = x.shape
    need = ctypes.c_size_t(0)
    _native.check("ws", _native.lib().kat_rational_bwd_workspace_size(rows, C, 1, G, code,
                                                                     dev.index, ctypes.byref(need)))
    ws = torch.empty(max(need.value, 16), dtype=torch.uint8, device=dev)
    dx, dn, dd = torch.empty_like(x), torch.empty(G, 6, device=dev), torch.empty(G, 4, device=dev)
    args = [x.data_ptr(), gy.data_ptr(), dx.data_ptr(), n.data_ptr(), d.data_ptr(),
            dn.data_ptr(), dd.data_ptr(), ws.data_ptr(), ws.numel(), rows, C, 1, G, code]
    if peers is not None:
        args.append(ctypes.byref(peers))
    args.append(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    st = lib_fn(*args)
    torch.cuda.synchronize()
    return st, dx, dn, dd


def _peers(buffers, rank, timeout_ms=2000, average=True):
    p = _native.KatPeers()
    p.world_size = len(buffers)
    p.rank = rank
    p.average = 1 if average else 0
    p.timeout_ms = timeout_ms
    for r, b in enumerate(buffers):
        p.buffers[r] = ctypes.c_void_p(b.data_ptr())
    return p


def test_world_one_matches_plain_backward(cuda_device):
    lib = _native.lib()
    G = 8
    x, gy, n, d = _problem(cuda_device, G=G)
    buf = torch.zeros(lib.kat_rational_exchange_buffer_bytes(G), dtype=torch.uint8,
                      device=cuda_device)
    st0, dx0, dn0, dd0 = _call(lib.kat_rational_bwd, x, gy, n, d, G)
    for _ in range(3):   # the epoch advances each call
        st1, dx1, dn1, dd1 = _call(lib.kat_rational_bwd_allreduce, x, gy, n, d, G,
                                   _peers([buf], 0))
        assert st0 == st1 == 0
        assert torch.equal(dx0, dx1) and torch.equal(dn0, dn1) and torch.equal(dd0, dd1)
    assert _native.device_status(0) == 0


def test_missing_rank_times_out_with_status(cuda_device):
    lib = _native.lib()
    G = 8
    x, gy, n, d = _problem(cuda_device, G=G)
    buf = torch.zeros(lib.kat_rational_exchange_buffer_bytes(G), dtype=torch.uint8,
                      device=cuda_device)
    _native.device_status(0, reset=True)
    st, dx, dn, dd = _call(lib.kat_rational_bwd_allreduce, x, gy, n, d, G,
                           _peers([buf, buf], 0, timeout_ms=50))
    assert st == 0
    assert _native.device_status(0, reset=True) == _native.KAT_DEVICE_EXCHANGE_TIMEOUT
    assert torch.isnan(dn).all() and torch.isnan(dd).all()
    _, dx_ref, dn_ref, _ = _call(lib.kat_rational_bwd, x, gy, n, d, G)
    assert torch.equal(dx, dx_ref)               # the elementwise part is unaffected
    assert torch.isfinite(dn_ref).all()           # and the context is still usable
    assert _native.device_status(0) == 0


def test_tag_out_of_step_is_refused_without_waiting(cuda_device):
    """A peer word tagged with a call out of step (here call 10 where call 1 or none is
    possible) cannot come from a correct pairing: the call writes NaN gradients, sets the
    status and marks the buffer broken, with no wait.  (Both "ranks" share one buffer; the
    first word of rank 1's row in the half of call 1 is preset.)"""
    lib = _native.lib()
    G = 8
    x, gy, n, d = _problem(cuda_device, G=G)
    buf = torch.zeros(lib.kat_rational_exchange_buffer_bytes(G), dtype=torch.uint8,
                      device=cuda_device)
    words = buf.view(torch.int64)
    n_words = 2 * G * 10                   # tagged words per rank row
    half_words = 8 * n_words               # rows of all KAT_MAX_PEERS ranks
    words[16 + half_words + n_words] = 10 << 32   # inbox at byte 128; half 1, rank 1, word 0
    _native.device_status(0, reset=True)
    st, dx, dn, dd = _call(lib.kat_rational_bwd_allreduce, x, gy, n, d, G,
                           _peers([buf, buf], 0, timeout_ms=60000))
    assert st == 0
    assert _native.device_status(0, reset=True) == _native.KAT_DEVICE_EXCHANGE_TIMEOUT
    assert torch.isnan(dn).all() and torch.isnan(dd).all()
    assert int(words[1]) == 1              # the broken word
    _, dx_ref, _, _ = _call(lib.kat_rational_bwd, x, gy, n, d, G)
    assert torch.equal(dx, dx_ref)


def test_broken_buffer_fails_at_once(cuda_device):
    """After a timeout the buffer is broken: the next call writes NaN gradients at once
    (no second wait) and stores nothing (the epoch does not advance)."""
    import time

    lib = _native.lib()
    G = 8
    x, gy, n, d = _problem(cuda_device, G=G)
    buf = torch.zeros(lib.kat_rational_exchange_buffer_bytes(G), dtype=torch.uint8,
                      device=cuda_device)
    words = buf.view(torch.int64)
    _native.device_status(0, reset=True)
    _call(lib.kat_rational_bwd_allreduce, x, gy, n, d, G, _peers([buf, buf], 0, timeout_ms=50))
    assert int(words[1]) == 1 and int(words[0]) == 1
    assert _native.device_status(0, reset=True) == _native.KAT_DEVICE_EXCHANGE_TIMEOUT
    t0 = time.time()
    st, dx, dn, dd = _call(lib.kat_rational_bwd_allreduce, x, gy, n, d, G,
                           _peers([buf, buf], 0, timeout_ms=20000))
    assert st == 0 and time.time() - t0 < 5.0
    assert torch.isnan(dn).all() and torch.isnan(dd).all()
    assert int(words[0]) == 1              # no new epoch was posted
    assert _native.device_status(0, reset=True) == _native.KAT_DEVICE_EXCHANGE_TIMEOUT
    assert _native.device_status(0) == 0


def test_exchange_grads_world_one_is_identity(cuda_device):
    """kat_rational_exchange_grads at world size 1: the rank-order sum of one rank is its
    own gradients, bit for bit, call after call (the epoch advances)."""
    lib = _native.lib()
    G = 8
    buf = torch.zeros(lib.kat_rational_exchange_buffer_bytes(G), dtype=torch.uint8,
                      device=cuda_device)
    g = torch.Generator(device="cpu").manual_seed(5)
    for call in range(3):
        dn = torch.randn(G, 6, generator=g).to(cuda_device)
        dd = torch.randn(G, 4, generator=g).to(cuda_device)
        dn0, dd0 = dn.clone(), dd.clone()
        p = _peers([buf], 0)
        st = lib.kat_rational_exchange_grads(dn.data_ptr(), dd.data_ptr(), G, ctypes.byref(p),
                                             ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
        assert st == 0 and torch.equal(dn, dn0) and torch.equal(dd, dd0)
    assert int(buf.view(torch.int64)[0]) == 3
    assert _native.device_status(0) == 0


def test_exchange_grads_missing_rank_gives_nan(cuda_device):
    lib = _native.lib()
    G = 4
    buf = torch.zeros(lib.kat_rational_exchange_buffer_bytes(G), dtype=torch.uint8,
                      device=cuda_device)
    dn = torch.ones(G, 6, device=cuda_device)
    dd = torch.ones(G, 4, device=cuda_device)
    _native.device_status(0, reset=True)
    p = _peers([buf, buf], 0, timeout_ms=50)
    st = lib.kat_rational_exchange_grads(dn.data_ptr(), dd.data_ptr(), G, ctypes.byref(p),
                                         ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert st == 0 and torch.isnan(dn).all() and torch.isnan(dd).all()
    assert _native.device_status(0, reset=True) == _native.KAT_DEVICE_EXCHANGE_TIMEOUT
    assert lib.kat_rational_exchange_grads(None, dd.data_ptr(), G, ctypes.byref(p), None) == \
        _native.KAT_ERR_NULL_POINTER


def test_descriptor_validation():
    lib = _native.lib()
    x = torch.empty(0)
    p = _native.KatPeers()
    p.world_size, p.rank, p.timeout_ms = 9, 0, 10
    st = lib.kat_rational_bwd_allreduce(None, None, None, 1, 1, 1, 1, None, 0, 0, 16, 1, 4, 0,
                                        ctypes.byref(p), None)
    assert st == _native.KAT_ERR_BAD_SHAPE
    p.world_size, p.rank = 2, 2
    st = lib.kat_rational_bwd_allreduce(None, None, None, 1, 1, 1, 1, None, 0, 0, 16, 1, 4, 0,
                                        ctypes.byref(p), None)
    assert st == _native.KAT_ERR_BAD_SHAPE
    del x


WORKER = r'''
import os, sys, datetime
sys.path.insert(0, {repo!r})
import torch, torch.distributed as dist
import rational_kat_cu_b200 as kat
rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
dev = torch.device("cuda", rank)
dist.init_process_group("nccl", rank=rank, world_size=world,
                        timeout=datetime.timedelta(seconds=60), device_id=dev)
g = torch.Generator().manual_seed(100 + rank)
x = torch.randn(6, 197, 768, generator=g).to(torch.bfloat16).to(dev)
gy = torch.randn(6, 197, 768, generator=g).to(torch.bfloat16).to(dev)
ref = kat.KAT_Group(num_groups=8, mode="gelu").to(dev)
m = kat.KAT_Group(num_groups=8, mode="gelu").to(dev)
m.enable_data_parallel(timeout_ms=5000)
for step in range(3):
    ref.zero_grad(); m.zero_grad()
    ref(x).backward(gy)
    m(x).backward(gy)
    local = torch.cat([ref.weight_numerator.grad.reshape(-1), ref.weight_denominator.grad.reshape(-1)])
    allg = [torch.empty_like(local) for _ in range(world)]
    dist.all_gather(allg, local)
    expect = sum(a.double() for a in allg) / world
    got = torch.cat([m.weight_numerator.grad.reshape(-1), m.weight_denominator.grad.reshape(-1)])
    torch.testing.assert_close(got.double(), expect, rtol=1e-5, atol=1e-5)
    gots = [torch.empty_like(got) for _ in range(world)]
    dist.all_gather(gots, got)
    assert all(torch.equal(gots[0], t) for t in gots), "ranks differ"
from rational_kat_cu_b200 import _native
from rational_kat_cu_b200.host_io import HostPipeline
# the host-buffer pipeline of a data-parallel module exchanges through the same buffers
hx = x.cpu().pin_memory(); hg = gy.cpu().pin_memory()
hy = torch.empty_like(hx).pin_memory(); hdx = torch.empty_like(hx).pin_memory()
for mod in (ref, m):
    mod.zero_grad(set_to_none=True)
    HostPipeline(mod, chunks=4).run(hx, hg, hy, hdx)
torch.cuda.synchronize()
local = torch.cat([ref.weight_numerator.grad.reshape(-1), ref.weight_denominator.grad.reshape(-1)])
allg = [torch.empty_like(local) for _ in range(world)]
dist.all_gather(allg, local)
expect = sum(a.double() for a in allg) / world
got = torch.cat([m.weight_numerator.grad.reshape(-1), m.weight_denominator.grad.reshape(-1)])
torch.testing.assert_close(got.double(), expect, rtol=1e-5, atol=1e-5)
gots = [torch.empty_like(got) for _ in range(world)]
dist.all_gather(gots, got)
assert all(torch.equal(gots[0], t) for t in gots), "pipeline ranks differ"
assert _native.device_status(rank) == 0
m.disable_data_parallel()      # collective teardown: unmap, barrier, free
assert m.exchange is None
dist.barrier()
dist.destroy_process_group()
print("rank", rank, "ok")
'''


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_two_gpu_exchange_matches_rank_order_average():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    code = WORKER.format(repo=REPO)
    procs = []
    for r in range(2):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE="2", LOCAL_RANK=str(r),
                   MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        procs.append(subprocess.Popen([sys.executable, "-c", code], env=env,
                                      stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True))
    outs = [p.communicate(timeout=240) for p in procs]
    for p, (so, se) in zip(procs, outs):
        assert p.returncode == 0 and "ok" in so, so + se[-3000:]
