"""The data-parallel gradient exchange protocol, restated on the CPU with ranks as threads
(tests/exchange_protocol.py restates kat_bwd_reduce_exchange_kernel in
rational_kat_cu_b200/csrc/kat_rational.cu).

Checked: under random skew every rank gets the same rank-order float64 sums of the same
call; a rank one call ahead writes the other inbox half while a slow rank still reads; a
reader never uses a row that is only partly written; a rank that stops makes the others time
out with NaN (bounded, no hang) and the failure is fail-stop (nothing stored afterwards); a
late rank gets either the right sums or NaN, never data of two calls mixed; a tag out of step
is refused.  Two planted protocol mistakes (one inbox half; one flag word per row instead of a
tag on every word) are shown to produce wrong sums in the same schedules.
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
    until rank 1 (fast) has posted its next call."""
    posted = threading.Event()
    waited = {}

    def hook(rank, epoch, point, peer):
        if rank == 1 and epoch == slow_epoch + 1 and point == "stored":
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
    """With one inbox half a fast rank's next call lands in the row a slow rank still reads
    or waits for: in the same schedule the slow rank no longer gets its call's sums (the
    words' tags turn the overwrite into a refused call or it reads the newer row)."""
    hook, waited = _ahead_schedule()
    results, _, _, alive = xp.run_ranks(2, {0: 6, 1: 6}, timeout_s=20.0, hook=hook,
                                        variant=xp.Variant(halves=1))
    assert not alive
    kinds = [xp.classify(v, 2, k) for k, v in enumerate(results[0], start=1)]
    assert kinds != ["exact"] * 6, kinds


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
        if rank == 0 and epoch == 5 and point == "stored":
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


def _half_written_schedule():
    """Rank 1 stops in the middle of writing its call-3 row into rank 0's inbox until rank 0
    has read that row (bounded, so a reader that correctly waits only delays the writer)."""
    read = threading.Event()

    def hook(rank, epoch, point, peer):
        if rank == 0 and epoch == 3 and point == "read" and peer == 1:
            read.set()
        if rank == 1 and epoch == 3 and point == "store_mid" and peer == 0:
            read.wait(2.0)

    return hook, read


def test_reader_waits_for_every_word_of_a_row():
    hook, read = _half_written_schedule()
    results, statuses, _, alive = xp.run_ranks(2, {0: 5, 1: 5}, timeout_s=20.0, hook=hook)
    assert not alive and all(s.value == 0 for s in statuses)
    _all_exact(results, 2)


def test_planted_row_flag_reads_a_half_written_row():
    """Checking one word per row (a flag) instead of every word's tag: the reader adds a row
    whose second half still holds the previous call's data."""
    hook, read = _half_written_schedule()
    results, _, _, alive = xp.run_ranks(2, {0: 5, 1: 5}, timeout_s=20.0, hook=hook,
                                        variant=xp.Variant(every_word=False))
    assert not alive and read.is_set()
    assert xp.classify(results[0][2], 2, 3) == "wrong"


def test_tag_out_of_step_is_refused():
    n = 10
    bufs = [xp.ExchangeBuffer(n) for _ in range(2)]
    # rank 1's row in the half of call 1 carries call 5's tag: out of step
    bufs[0].inbox[1][1] = xp.encode(xp.contribution(1, 5, n), 5)
    st = xp.Status()
    out = xp.exchange_call(0, 2, bufs, xp.contribution(0, 1, n), 5.0, st)
    assert xp.is_nan(out) and st.value == 2 and bufs[0].broken == 1
    # One call ahead is the normal case of a fast peer: its call 2 sits in the other half.
    bufs = [xp.ExchangeBuffer(n) for _ in range(2)]
    bufs[0].inbox[1][1] = xp.encode(xp.contribution(1, 1, n), 1)
    bufs[0].inbox[0][1] = xp.encode(xp.contribution(1, 2, n), 2)
    st = xp.Status()
    out = xp.exchange_call(0, 2, bufs, xp.contribution(0, 1, n), 5.0, st)
    assert xp.classify(out, 2, 1) == "exact" and st.value == 0


def test_words_round_trip_every_bit():
    v = np.array([0.0, -0.0, 1.5, -3.25e300, 5e-324, np.inf, -np.inf, 1.0 / 3.0])
    w = xp.encode(v, 7)
    assert all(t == 7 and 0 <= d < 2 ** 32 for t, d in w)
    back = xp.decode(w)
    assert back.tobytes() == v.tobytes()
