"""CPU restatement of the data-parallel gradient exchange protocol (test infrastructure).

Restates, step for step, what `kat_bwd_reduce_exchange_kernel`
(rational_kat_cu_b200/csrc/kat_rational.cu) does with the exchange buffers once its block
has this GPU's G x 10 fp64 sums, so the protocol can be run on the CPU with simulated ranks
(threads) and any interleaving a test forces:

  1. a buffer marked broken by an earlier failure: NaN at once, nothing stored anywhere;
  2. epoch = own epoch + 1 (kernel-owned counter); tag = epoch mod 2^32; half = epoch & 1;
  3. store this rank's sums into row `rank` of that half in every rank's inbox, each fp64
     as two words (tag, low 32 bits) and (tag, high 32 bits) — one word is one single-copy
     atomic 8-byte store on the GPU, one tuple assignment here;
  4. wait, bounded by the timeout, until every word of every row of the half on this rank
     carries the tag; a word may meanwhile only carry the tag of call epoch - 2 (or 0 before
     the first two calls): any other tag is out of step;
  5. on a timeout or a tag out of step: mark the own buffer broken and return NaN;
  6. otherwise decode the rows and add them in rank order in float64.

Ranks here share one address space and the GIL orders every access, which is at least as
strong as the kernel's relaxed system-scope word stores and loads.  `Variant` plants
protocol mistakes (one inbox half instead of two; no fail-stop and no step check; only the
first word of a row checked, as a single flag would be) so the tests can show they would be
caught.  Nothing in the product imports this file.
"""

from __future__ import annotations

import dataclasses
import struct
import threading
import time
from typing import Callable, Dict, List, Optional, Tuple

import numpy as np

MAX_PEERS = 8
NAN = float("nan")
MASK32 = 0xFFFFFFFF


@dataclasses.dataclass
class Variant:
    halves: int = 2             # 1 plants the overwrite race the two halves prevent
    fail_stop: bool = True      # False plants "keep posting after a timeout, no step check"
    every_word: bool = True     # False plants "wait for the first word of a row only"


Word = Tuple[int, int]          # (tag, 32 payload bits)


def encode(values: np.ndarray, tag: int) -> List[Word]:
    words: List[Word] = []
    for v in values:
        bits = struct.unpack("<Q", struct.pack("<d", float(v)))[0]
        words.append((tag, bits & MASK32))
        words.append((tag, bits >> 32))
    return words


def decode(words: List[Word]) -> np.ndarray:
    out = np.empty(len(words) // 2, dtype=np.float64)
    for i in range(out.shape[0]):
        bits = words[2 * i][1] | (words[2 * i + 1][1] << 32)
        out[i] = struct.unpack("<d", struct.pack("<Q", bits))[0]
    return out


class ExchangeBuffer:
    """One rank's exchange buffer: epoch, broken word, inbox[2][MAX_PEERS][2n] words."""

    def __init__(self, n: int):
        self.epoch = 0
        self.broken = 0
        self.inbox = [[[(0, 0)] * (2 * n) for _ in range(MAX_PEERS)] for _ in range(2)]
        self.stores_from: List[int] = []   # ranks that stored into this buffer, in order


class Status:
    """Stand-in for the sticky device status word of one rank."""

    def __init__(self):
        self.value = 0


Hook = Callable[[int, int, str, int], None]   # (rank, epoch, point, peer or word index)


def exchange_call(rank: int, world: int, bufs: List[ExchangeBuffer], sums: np.ndarray,
                  timeout_s: float, status: Status, hook: Optional[Hook] = None,
                  variant: Variant = Variant(), poll_s: float = 1e-4) -> np.ndarray:
    """One call of the exchange on rank `rank`; returns the rank-order float64 totals, or an
    all-NaN vector when the call failed (steps 1-6 above)."""
    hook = hook or (lambda *a: None)
    own = bufs[rank]
    n = sums.shape[0]
    if variant.fail_stop and own.broken:
        status.value = 2
        return np.full(n, NAN)
    own.epoch += 1
    epoch = own.epoch
    tag = epoch & MASK32
    stale = (epoch - 2) & MASK32
    half = epoch & 1 if variant.halves == 2 else 0
    words = encode(sums, tag)
    for r in range(world):
        hook(rank, epoch, "store", r)
        row = bufs[r].inbox[half][rank]
        for i, w in enumerate(words):
            if i == len(words) // 2:
                hook(rank, epoch, "store_mid", r)
            row[i] = w
        bufs[r].stores_from.append(rank)
    hook(rank, epoch, "stored", -1)
    t0 = time.monotonic()
    ok = True
    for q in range(world):
        row = own.inbox[half][q]
        for i in range(2 * n if variant.every_word else 1):
            while True:
                t = row[i][0]
                if t == tag:
                    break
                in_step = t == stale or (epoch <= 2 and t == 0) or not variant.fail_stop
                if not in_step or time.monotonic() - t0 > timeout_s:
                    ok = False
                    break
                time.sleep(poll_s)
            if not ok:
                break
        if not ok:
            break
    if not ok:
        if variant.fail_stop:
            own.broken = 1
        status.value = 2
        return np.full(n, NAN)
    tot = np.zeros(n, dtype=np.float64)
    for q in range(world):
        hook(rank, epoch, "read", q)
        tot = tot + decode(own.inbox[half][q])
    return tot


def contribution(rank: int, call: int, n: int) -> np.ndarray:
    """Rank `rank`'s G x 10 sums at its call number `call` (1-based): distinct per call."""
    rng = np.random.default_rng(1000 * call + rank)
    return rng.standard_normal(n) * (1.0 + call)


def expected(world: int, call: int, n: int) -> np.ndarray:
    tot = np.zeros(n, dtype=np.float64)
    for q in range(world):
        tot = tot + contribution(q, call, n)
    return tot


def run_ranks(world: int, calls: Dict[int, int], n: int = 40, timeout_s: float = 1.0,
              hook: Optional[Hook] = None, variant: Variant = Variant(),
              join_s: float = 60.0):
    """Run `calls[r]` exchange calls on each rank r in its own thread.  Returns
    (results[r] = list of totals per call, statuses, buffers, threads still alive)."""
    bufs = [ExchangeBuffer(n) for _ in range(world)]
    statuses = [Status() for _ in range(world)]
    results: List[List[np.ndarray]] = [[] for _ in range(world)]
    errors: List[BaseException] = []

    def body(r):
        try:
            for k in range(1, calls[r] + 1):
                results[r].append(exchange_call(r, world, bufs, contribution(r, k, n),
                                                timeout_s, statuses[r], hook, variant))
        except BaseException as e:  # surfaced to the test
            errors.append(e)

    threads = [threading.Thread(target=body, args=(r,), daemon=True) for r in range(world)]
    for t in threads:
        t.start()
    deadline = time.monotonic() + join_s
    for t in threads:
        t.join(max(0.0, deadline - time.monotonic()))
    alive = [i for i, t in enumerate(threads) if t.is_alive()]
    if errors:
        raise errors[0]
    return results, statuses, bufs, alive


def is_nan(v: np.ndarray) -> bool:
    return bool(np.all(np.isnan(v)))


def exact(v: np.ndarray, want: np.ndarray) -> bool:
    return bool(np.array_equal(v, want))


def classify(v: np.ndarray, world: int, call: int) -> str:
    """'exact' (the rank-order sum of call `call`), 'nan' (a reported failure) or 'wrong'."""
    if is_nan(v):
        return "nan"
    if exact(v, expected(world, call, v.shape[0])):
        return "exact"
    return "wrong"


__all__ = ["Variant", "ExchangeBuffer", "Status", "exchange_call", "contribution", "expected",
           "run_ranks", "classify", "is_nan", "exact", "encode", "decode"]
