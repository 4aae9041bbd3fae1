"""Data-parallel host logic on CPU ranks (gloo, world size 2): the coefficient-gradient
exchange gives every rank the same, rank-order-summed gradients; a data-parallel step over
batch shards reproduces the single-process gradients; a rank that dies before the exchange
makes the survivor fail with an error instead of hanging."""

import os
import socket
import subprocess
import sys
import tempfile

import pytest
import torch

from rational_kat_cu_b200.distributed import shard_rows

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


WORKER = r'''
import os, sys, datetime
sys.path.insert(0, {repo!r})
import torch, torch.distributed as dist
import rational_kat_cu_b200 as kat
from rational_kat_cu_b200.distributed import allreduce_coefficient_grads, shard_rows
rank, world, mode, out = int(sys.argv[1]), int(sys.argv[2]), sys.argv[3], sys.argv[4]
dist.init_process_group("gloo", init_method="tcp://127.0.0.1:{port}", rank=rank,
                        world_size=world, timeout=datetime.timedelta(seconds=6))
torch.manual_seed(0)
x = torch.randn(8, 5, 32)
gy = torch.randn(8, 5, 32)
m = kat.KAT_Group(num_groups=4, mode="gelu", device="cpu")
if mode == "exchange":
    m.weight_numerator.grad = torch.full((1, 6), float(rank + 1)) / 3.0
    m.weight_denominator.grad = torch.arange(16.0).view(4, 4) * (rank + 1) / 7.0
    allreduce_coefficient_grads(m, average=True)
elif mode == "step":
    sl = shard_rows(x.shape[0], rank, world)
    y = m(x[sl])
    y.backward(gy[sl])
    allreduce_coefficient_grads(m, average=False)
elif mode == "dead_peer":
    if rank == 1:
        os._exit(0)
    m.weight_numerator.grad = torch.ones(1, 6)
    m.weight_denominator.grad = torch.ones(4, 4)
    try:
        allreduce_coefficient_grads(m)
        print("NO-ERROR")
    except Exception as e:
        print("RAISED", type(e).__name__)
    os._exit(0)
elif mode.startswith("teardown"):
    import json, time
    from rational_kat_cu_b200.distributed import PeerExchange

    class FakeLib:
        """Records the exchange-buffer calls with a system-wide monotonic time stamp."""
        def __init__(self):
            self.log = []
        def kat_rational_exchange_close(self, ptr):
            self.log.append(("close", ptr.value, time.monotonic()))
            return 0
        def kat_rational_exchange_destroy(self, ptr):
            self.log.append(("destroy", ptr.value, time.monotonic()))
            return 0

    pe = PeerExchange.__new__(PeerExchange)
    pe._lib = FakeLib()
    lib = pe._lib
    pe._opened = [1000 + r for r in range(world) if r != rank]
    pe._local = 2000 + rank
    pe.group = None
    pe.device = torch.device("cpu")
    raised = None
    if mode == "teardown":
        if rank == 1:
            time.sleep(1.0)        # a slow rank: the others must not free before it unmapped
        pe.close()
        pe.close()                 # idempotent
    elif mode == "teardown_gc":
        del pe
    elif mode == "teardown_dead":
        if rank == 1:
            os._exit(0)
        try:
            pe.close()
        except Exception as e:
            raised = type(e).__name__
    with open(f"{{out}}.{{rank}}.json", "w") as fh:
        json.dump({{"log": lib.log, "raised": raised}}, fh)
    os._exit(0)
torch.save({{"num": m.weight_numerator.grad, "den": m.weight_denominator.grad}},
           f"{{out}}.{{rank}}.pt")
dist.destroy_process_group()
'''


def run_ranks(mode, world=2, timeout=120):
    port = free_port()
    code = WORKER.format(repo=REPO, port=port)
    with tempfile.TemporaryDirectory() as td:
        out = os.path.join(td, "grads")
        env = dict(os.environ, MASTER_ADDR="127.0.0.1")
        procs = [subprocess.Popen([sys.executable, "-c", code, str(r), str(world), mode, out],
                                  stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True,
                                  env=env) for r in range(world)]
        outs = []
        for p in procs:
            try:
                so, se = p.communicate(timeout=timeout)
            except subprocess.TimeoutExpired:
                p.kill()
                so, se = p.communicate()
                raise AssertionError(f"rank timed out: {se[-2000:]}")
            outs.append((p.returncode, so, se))
        results = {}
        for r in range(world):
            path = f"{out}.{r}.pt"
            if os.path.exists(path):
                results[r] = torch.load(path)
            path = f"{out}.{r}.json"
            if os.path.exists(path):
                import json

                with open(path) as fh:
                    results[r] = json.load(fh)
        return outs, results


def test_exchange_is_identical_on_every_rank():
    outs, res = run_ranks("exchange")
    assert all(rc == 0 for rc, _, _ in outs), outs
    assert torch.equal(res[0]["num"], res[1]["num"])
    assert torch.equal(res[0]["den"], res[1]["den"])
    expect_num = (torch.full((1, 6), 1.0) / 3.0 + torch.full((1, 6), 2.0) / 3.0) / 2
    torch.testing.assert_close(res[0]["num"], expect_num)
    expect_den = (torch.arange(16.0).view(4, 4) / 7.0 + torch.arange(16.0).view(4, 4) * 2 / 7.0) / 2
    torch.testing.assert_close(res[0]["den"], expect_den)


def test_sharded_step_matches_single_process():
    outs, res = run_ranks("step")
    assert all(rc == 0 for rc, _, _ in outs), outs
    import rational_kat_cu_b200 as kat

    torch.manual_seed(0)
    x = torch.randn(8, 5, 32)
    gy = torch.randn(8, 5, 32)
    m = kat.KAT_Group(num_groups=4, mode="gelu", device="cpu")
    m(x).backward(gy)
    torch.testing.assert_close(res[0]["num"], m.weight_numerator.grad, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(res[0]["den"], m.weight_denominator.grad, rtol=1e-5, atol=1e-5)
    assert torch.equal(res[0]["num"], res[1]["num"])


def test_dead_peer_raises_instead_of_hanging():
    outs, _ = run_ranks("dead_peer", timeout=90)
    rc0, so0, se0 = outs[0]
    assert "RAISED" in so0, so0 + se0


@pytest.mark.parametrize("rows,world", [(10, 3), (8, 8), (3, 4), (0, 2)])
def test_shard_rows_partition(rows, world):
    seen = []
    for r in range(world):
        sl = shard_rows(rows, r, world)
        seen.extend(range(rows)[sl])
    assert seen == list(range(rows))


def test_peer_exchange_teardown_frees_only_after_every_rank_unmapped():
    """close() is collective: each rank unmaps the peers' buffers, all meet at a barrier, and
    only then does any rank free its own buffer, even when one rank is a second late."""
    outs, res = run_ranks("teardown")
    assert all(rc == 0 for rc, _, _ in outs), outs
    closes = [t for r in res for op, _, t in res[r]["log"] if op == "close"]
    destroys = [t for r in res for op, _, t in res[r]["log"] if op == "destroy"]
    assert len(closes) == 2 and len(destroys) == 2       # one peer each; second close() no-op
    assert min(destroys) > max(closes)
    for r in res:
        assert [e[1] for e in res[r]["log"] if e[0] == "destroy"] == [2000 + r]


def test_peer_exchange_garbage_collection_unmaps_but_never_frees():
    outs, res = run_ranks("teardown_gc")
    assert all(rc == 0 for rc, _, _ in outs), outs
    for r in res:
        assert [e[0] for e in res[r]["log"]] == ["close"]


def test_peer_exchange_teardown_with_a_dead_rank_raises_and_keeps_the_buffer():
    outs, res = run_ranks("teardown_dead", timeout=90)
    assert res[0]["raised"] is not None
    assert [e[0] for e in res[0]["log"]] == ["close"]
