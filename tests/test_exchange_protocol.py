"""The data-parallel gradient exchange protocol, restated on the CPU with ranks as threads
(tests/exchange_protocol.py restates kat_bwd_reduce_exchange_kernel in
rational_kat_cu_b200/csrc/kat_rational.cu).

Checked: under random skew every rank gets the same rank-order float64 sums of the same
call; a rank one call ahead writes the other inbox half while a slow rank still reads; a
rank that stops makes the others time out with NaN (bounded, no hang) and the failure is
fail-stop; a late rank gets either the right sums or NaN, never data of two calls mixed; a
flag more than one call ahead is refused.  Two planted protocol mistakes (one inbox half;
no fail-stop) are shown to produce wrong sums in the same schedules.
"""

import random
import threading
import time

import numpy as np
import pytest

import exchange_protocol as xp


def _all_exact(results, world):
    for r in range(world):
        for k, v in enumerate(results[r], start=1):
            assert xp.classify(v, world, k) == "exact", (r, k)
    for k in range(len(results[0])):
        for r in range(1, world):
            assert np.array_equal(results[r][k], results[0][k])


@pytest.mark.parametrize("world", [2, 3, 4, 8])
def test_random_skew_gives_identical_rank_order_sums(world):
    rngs = {r: random.Random(17 + r) for r in range(world)}
    lock = threading.Lock()

    def jitter(rank, epoch, point, peer):
        with lock:
            d = rngs[rank].random()
        if d < 0.3:
            time.sleep(d * 4e-3)

    calls = {r: 25 for r in range(world)}
    results, statuses, _, alive = xp.run_ranks(world, calls, timeout_s=20.0, hook=jitter)
    assert not alive
    assert all(s.value == 0 for s in statuses)
    _all_exact(results, world)


def _ahead_schedule(slow_epoch=3):
    """Rank 0 (slow) reads its call-`slow_epoch` inbox; between its row 0 and row 1 it waits
    until rank 1 (fast) has posted its next call (data and flag)."""
    posted = threading.Event()
    waited = {}

    def hook(rank, epoch, point, peer):
        if rank == 1 and epoch == slow_epoch + 1 and point == "flagged":
            posted.set()
        if rank == 0 and epoch == slow_epoch and point == "read" and peer == 1:
            waited["ok"] = posted.wait(10.0)

    return hook, waited


def test_rank_one_call_ahead_does_not_disturb_a_slow_reader():
    hook, waited = _ahead_schedule()
    results, statuses, _, alive = xp.run_ranks(2, {0: 6, 1: 6}, timeout_s=20.0, hook=hook)
    assert not alive and waited.get("ok") is True
    assert all(s.value == 0 for s in statuses)
    _all_exact(results, 2)


def test_planted_single_half_is_caught():
    """With one inbox half the fast rank's next call overwrites the row the slow rank is
    about to add: the same schedule then yields a wrong sum."""
    hook, waited = _ahead_schedule()
    results, _, _, alive = xp.run_ranks(2, {0: 6, 1: 6}, timeout_s=20.0, hook=hook,
                                        variant=xp.Variant(halves=1))
    assert not alive and waited.get("ok") is True
    assert xp.classify(results[0][2], 2, 3) == "wrong"


def test_stopped_rank_times_out_with_nan_and_fail_stop():
    world, timeout = 3, 0.3
    t0 = time.monotonic()
    results, statuses, bufs, alive = xp.run_ranks(world, {0: 6, 1: 6, 2: 3}, timeout_s=timeout)
    elapsed = time.monotonic() - t0
    assert not alive
    assert elapsed < 10 * timeout + 5.0          # bounded: one timeout per waiting rank
    for r in (0, 1):
        kinds = [xp.classify(v, world, k) for k, v in enumerate(results[r], start=1)]
        assert kinds == ["exact"] * 3 + ["nan"] * 3, (r, kinds)
        assert statuses[r].value == 2 and bufs[r].broken == 1
    assert [xp.classify(v, world, k) for k, v in enumerate(results[2], start=1)] == ["exact"] * 3
    # After the failed call 4 nothing more is stored anywhere: 4 stores from ranks 0 and 1
    # (calls 1-4) and 3 from rank 2 in every buffer.
    for b in bufs:
        assert b.stores_from.count(0) == 4 and b.stores_from.count(1) == 4
        assert b.stores_from.count(2) == 3


def _late_schedule(timeout):
    """Rank 1 reaches its call 3 late: it waits (bounded) until rank 0 has posted call 5, or
    long enough for rank 0's call 3 to have timed out."""
    far_ahead = threading.Event()

    def hook(rank, epoch, point, peer):
        if rank == 0 and epoch == 5 and point == "flagged":
            far_ahead.set()
        if rank == 1 and epoch == 3 and point == "store" and peer == 0:
            far_ahead.wait(4 * timeout + 1.0)

    return hook, far_ahead


def test_late_rank_gets_right_sums_or_nan_never_mixed():
    world, timeout = 2, 0.3
    hook, far_ahead = _late_schedule(timeout)
    results, statuses, bufs, alive = xp.run_ranks(world, {0: 5, 1: 5}, timeout_s=timeout,
                                                  hook=hook)
    assert not alive
    assert not far_ahead.is_set()         # rank 0 stopped posting after its failure
    for r in range(world):
        kinds = [xp.classify(v, world, k) for k, v in enumerate(results[r], start=1)]
        assert "wrong" not in kinds, (r, kinds)
        assert kinds[:2] == ["exact", "exact"]
        assert kinds[-1] == "nan" and statuses[r].value == 2
    assert [xp.classify(v, world, 3) for v in results[0][2:3]] == ["nan"]


def test_planted_no_fail_stop_mixes_calls():
    """Without fail-stop the timed-out rank keeps posting: two calls later it writes the
    half the late rank then reads, and the late rank adds data of another call."""
    world, timeout = 2, 0.3
    hook, far_ahead = _late_schedule(timeout)
    results, _, _, alive = xp.run_ranks(world, {0: 5, 1: 5}, timeout_s=timeout, hook=hook,
                                        variant=xp.Variant(fail_stop=False))
    assert not alive and far_ahead.is_set()
    assert xp.classify(results[1][2], world, 3) == "wrong"


def test_flag_more_than_one_call_ahead_is_refused():
    n = 10
    bufs = [xp.ExchangeBuffer(n) for _ in range(2)]
    bufs[0].flags[1] = 5                       # rank 1 seen at call 5 before rank 0's call 1
    st = xp.Status()
    out = xp.exchange_call(0, 2, bufs, xp.contribution(0, 1, n), 5.0, st)
    assert xp.is_nan(out) and st.value == 2 and bufs[0].broken == 1
    # One call ahead is the normal case of a fast peer and is accepted.
    bufs = [xp.ExchangeBuffer(n) for _ in range(2)]
    bufs[0].flags[1] = 2
    bufs[0].inbox[1, 1, :] = xp.contribution(1, 1, n)
    st = xp.Status()
    out = xp.exchange_call(0, 2, bufs, xp.contribution(0, 1, n), 5.0, st)
    assert xp.classify(out, 2, 1) == "exact" and st.value == 0
