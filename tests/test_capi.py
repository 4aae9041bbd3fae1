"""The C ABI library on the CPU: it loads, exports every symbol include/*.h declares, rejects bad arguments before touching a GPU, and its launch geometry covers every
element exactly once with a consistent partial-sum layout (checked by a host-side
restatement of the kernels' index arithmetic)."""

import ctypes
import os
import re

import pytest

from rational_kat_cu_b200 import _native

INCLUDE = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include")


def declared_functions():
    names = set()
    for h in sorted(os.listdir(INCLUDE)):
        if h.endswith(".h"):
            text = re.sub(r"/\*.*?\*/", "", open(os.path.join(INCLUDE, h)).read(), flags=re.S)
            names |= set(re.findall(r"\b(kat_\w+)\s*\(", text))
    return sorted(names)


def test_header_declares_expected_entry_points():
    assert declared_functions() == sorted(_native.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol():
    lib = _native.lib()
    raw = ctypes.CDLL(_native.library_path())
    for name in declared_functions():
        assert hasattr(raw, name), f"{name} not exported"
    assert lib.kat_rational_abi_version() == _native.ABI_VERSION


def test_strerror_covers_every_status():
    texts = {code: _native.strerror(code) for code in range(0, 7)}
    assert texts[0] == "success"
    assert len(set(texts.values())) == 7
    assert "unknown" in _native.strerror(99)


def test_bspline_entry_points_validate_before_launch():
    lib = _native.lib()
    E = _native
    for nk, order in ((15, 0), (15, 6), (4, 3), (65, 3)):
        assert lib.kat_bspline_basis_fwd(1, 1, 1, 4, 8, nk, order, None) == E.KAT_ERR_BAD_SHAPE
        assert lib.kat_bspline_basis_bwd(1, 1, 1, 1, 4, 8, nk, order, None) == E.KAT_ERR_BAD_SHAPE
    assert lib.kat_bspline_basis_fwd(1, 1, 1, -1, 8, 15, 3, None) == E.KAT_ERR_BAD_SHAPE
    assert lib.kat_bspline_basis_fwd(None, 1, 1, 4, 8, 15, 3, None) == E.KAT_ERR_NULL_POINTER
    assert lib.kat_bspline_basis_bwd(1, 1, None, 1, 4, 8, 15, 3, None) == E.KAT_ERR_NULL_POINTER
    # empty problems are a successful no-op
    assert lib.kat_bspline_basis_fwd(None, None, None, 0, 8, 15, 3, None) == E.KAT_OK
    assert lib.kat_bspline_basis_bwd(None, None, None, None, 4, 0, 15, 3, None) == E.KAT_OK


def test_formula_entry_points_validate_before_launch():
    lib = _native.lib()
    assert _native.KAT_FORMULA_KAT == 0 and _native.KAT_FORMULA_ABS_SUM == 1
    for bad in (-1, 2, 99):
        assert lib.kat_rational_fwd_formula(1, 1, 1, 1, 4, 16, 1, 4, 0, bad, None) == \
            _native.KAT_ERR_BAD_FORMULA
        assert lib.kat_rational_bwd_formula(1, 1, 1, 1, 1, 1, 1, 1, 1 << 20, 4, 16, 1, 4, 0, bad,
                                            None) == _native.KAT_ERR_BAD_FORMULA
    # the other argument checks come first, exactly as for the KAT entry points
    assert lib.kat_rational_fwd_formula(1, 1, 1, 1, 4, 18, 1, 4, 0, 1, None) == \
        _native.KAT_ERR_BAD_GROUPS
    assert lib.kat_rational_bwd_formula(1, 1, 1, 1, 1, None, 1, 1, 1 << 20, 4, 16, 1, 4, 0, 1,
                                        None) == _native.KAT_ERR_NULL_POINTER
    assert lib.kat_rational_fwd_formula(None, None, 1, 1, 0, 16, 1, 4, 0, 1, None) == _native.KAT_OK
    assert "formula" in _native.strerror(_native.KAT_ERR_BAD_FORMULA)


def test_gemm_entry_points_validate_before_launch():
    lib = _native.lib()
    E = _native
    P = 16  # an aligned address value; every call below has a bad argument, so none is used
    for m, n, k in ((-1, 256, 64), (128, 255, 64), (128, 256, 63), (128, 0, 64),
                    (1 << 31, 256, 64), (128, 256, 0)):
        assert lib.kat_gemm_bf16(P, P, None, P, m, n, k, None) == E.KAT_ERR_BAD_SHAPE
        assert lib.kat_gemm_rational_fwd(P, P, None, P, P, P, P, m, n, k, 8, 0, None) == \
            E.KAT_ERR_BAD_SHAPE
        assert lib.kat_gemm_rational_bwd(P, P, P, P, P, P, P, P, P, 1 << 20, m, n, k, 8, 0,
                                         None) == E.KAT_ERR_BAD_SHAPE
        assert lib.kat_gemm_rational_bwd_workspace_bytes(m, n, 8, 0) == 0
    assert lib.kat_gemm_bf16(None, P, None, P, 128, 256, 64, None) == E.KAT_ERR_NULL_POINTER
    assert lib.kat_gemm_rational_fwd(P, P, None, None, P, P, P, 128, 256, 64, 8, 0, None) == \
        E.KAT_ERR_NULL_POINTER
    assert lib.kat_gemm_rational_bwd(P, P, P, P, P, P, None, P, P, 1 << 20, 128, 256, 64, 8, 0,
                                     None) == E.KAT_ERR_NULL_POINTER
    # groups: N / G must be a whole multiple of the 32-column epilogue chunk
    for g in (0, -1, 3, 16):
        assert lib.kat_gemm_rational_fwd(P, P, None, P, P, P, P, 128, 256, 64, g, 0, None) == \
            E.KAT_ERR_BAD_GROUPS
        assert lib.kat_gemm_rational_bwd(P, P, P, P, P, P, P, P, P, 1 << 20, 128, 256, 64, g, 0,
                                         None) == E.KAT_ERR_BAD_GROUPS
    for f in (-1, 2):
        assert lib.kat_gemm_rational_fwd(P, P, None, P, P, P, P, 128, 256, 64, 8, f, None) == \
            E.KAT_ERR_BAD_FORMULA
    # an empty problem is a successful no-op (nothing is enqueued for the forward)
    assert lib.kat_gemm_bf16(P, P, None, P, 0, 256, 64, None) == E.KAT_OK
    assert lib.kat_gemm_rational_fwd(P, P, None, P, P, P, P, 0, 256, 64, 8, 0, None) == E.KAT_OK
    # TMA needs 16-byte aligned operands
    assert lib.kat_gemm_bf16(P + 2, P, None, P, 128, 256, 64, None) == E.KAT_ERR_BAD_SHAPE
    assert lib.kat_gemm_bf16(P, P, P + 8, P, 128, 256, 64, None) == E.KAT_ERR_BAD_SHAPE


def _fwd(x=1, y=1, num=1, den=1, batch=4, channels=16, inner=1, groups=4, dtype=0):
    return _native.lib().kat_rational_fwd(x, y, num, den, batch, channels, inner, groups, dtype,
                                          None)


def _bwd(x=1, gy=1, dx=1, num=1, den=1, dn=1, dd=1, ws=1, ws_bytes=1 << 20, batch=4,
         channels=16, inner=1, groups=4, dtype=0):
    return _native.lib().kat_rational_bwd(x, gy, dx, num, den, dn, dd, ws, ws_bytes, batch,
                                          channels, inner, groups, dtype, None)


def test_argument_errors_return_before_any_launch():
    assert _fwd(dtype=7) == _native.KAT_ERR_BAD_DTYPE
    assert _fwd(channels=18, groups=4) == _native.KAT_ERR_BAD_GROUPS
    assert _fwd(groups=0) == _native.KAT_ERR_BAD_GROUPS
    assert _fwd(batch=-1) == _native.KAT_ERR_BAD_SHAPE
    assert _fwd(inner=-3) == _native.KAT_ERR_BAD_SHAPE
    assert _fwd(batch=1 << 40, channels=1 << 12, groups=1) == _native.KAT_ERR_BAD_SHAPE
    assert _fwd(x=None) == _native.KAT_ERR_NULL_POINTER
    assert _fwd(num=None) == _native.KAT_ERR_NULL_POINTER
    # Empty problems are a successful no-op (nothing is enqueued).
    assert _fwd(x=None, y=None, batch=0) == _native.KAT_OK
    assert _bwd(dn=None) == _native.KAT_ERR_NULL_POINTER
    assert _bwd(gy=None) == _native.KAT_ERR_NULL_POINTER
    assert _bwd(dtype=3) == _native.KAT_ERR_BAD_DTYPE
    out = ctypes.c_size_t(123)
    lib = _native.lib()
    assert lib.kat_rational_bwd_workspace_size(4, 18, 1, 4, 0, 0, ctypes.byref(out)) == \
        _native.KAT_ERR_BAD_GROUPS
    assert lib.kat_rational_bwd_workspace_size(0, 16, 1, 4, 0, 0, ctypes.byref(out)) == \
        _native.KAT_OK and out.value == 0
    assert lib.kat_rational_bwd_workspace_size(4, 16, 1, 4, 0, 0, None) == \
        _native.KAT_ERR_NULL_POINTER


# ---------------------------------------------------------------------------
# Host restatement of the kernels' work decomposition.
# ---------------------------------------------------------------------------

def block_items(p, blk):
    """Item range of block `blk`: an even split of all items, or (col_block_blocks > 0) an
    even split of one column block's rows over that column block's blocks."""
    cq = p["col_block_blocks"]
    if cq == 0:
        q, r = divmod(p["items"], p["blocks"])
        i0 = blk * q + min(blk, r)
        return i0, i0 + q + (1 if blk < r else 0)
    cr = p["col_block_extra"]
    counts = [cq + 1] * cr + [cq] * (p["col_blocks"] - cr)
    first = 0
    for cb, n in enumerate(counts):
        if blk < first + n:
            k = blk - first
            q, r = divmod(p["rows"], n)
            i0 = cb * p["rows"] + k * q + min(k, r)
            return i0, i0 + q + (1 if k < r else 0)
        first += n
    raise AssertionError(f"block {blk} beyond the split")


def simulate(p):
    """Element coverage and partial-slot writes/reads, following kat_fwd_kernel /
    kat_bwd_kernel / kat_bwd_reduce_kernel index arithmetic."""
    rows, vec = p["rows"], p["vec"]
    vec_cols = p["width"] // vec
    vec_group = p["group_width"] // vec
    tc, tr = p["tile_cols"], p["tile_rows"]
    covered = {}
    written = {}
    for blk in range(p["blocks"]):
        i0, i1 = block_items(p, blk)
        cb0 = i0 // rows
        i = i0
        while i < i1:
            cb = i // rows
            seg_end = min(i1, (cb + 1) * rows)
            for t in range(p["threads"]):
                c, r_off = t % tc, t // tc
                col = cb * tc + c
                if r_off >= tr or col >= vec_cols:
                    continue
                r = i - cb * rows + r_off
                while r < seg_end - cb * rows:
                    key = (r, col)
                    covered[key] = covered.get(key, 0) + 1
                    r += tr
            col0 = cb * tc
            col_end = min(col0 + tc, vec_cols)
            g_first, g_last = col0 // vec_group, (col_end - 1) // vec_group
            seg = cb - cb0
            assert seg < p["max_segments"]
            for lg in range(g_last - g_first + 1):
                assert lg < p["max_local_groups"]
                slot = (blk, seg, lg)
                assert slot not in written
                written[slot] = g_first + lg
            i = seg_end
    read = {}
    for g in range(p["num_groups"]):
        for blk in range(p["blocks"]):
            i0, i1 = block_items(p, blk)
            cb0, cb1 = i0 // rows, (i1 - 1) // rows
            for cb in range(cb0, cb1 + 1):
                col0 = cb * tc
                col_end = min(col0 + tc, vec_cols)
                g_first, g_last = col0 // vec_group, (col_end - 1) // vec_group
                if g < g_first:
                    break
                if g > g_last:
                    continue
                slot = (blk, cb - cb0, g - g_first)
                assert written.get(slot) == g, (slot, g)
                read[slot] = read.get(slot, 0) + 1
    return covered, written, read


SHAPES = [
    # batch, channels, inner, groups, dtype, sms, occupancy
    (37, 96, 1, 8, 0, 7, 3),
    (5, 3072, 1, 8, 2, 3, 2),
    (9, 768, 1, 64, 2, 4, 1),        # 12-wide groups: 8-element vectors do not fit
    (3, 8192, 1, 64, 0, 2, 2),       # several column blocks per row
    (4, 16, 49, 8, 0, 5, 2),         # NCHW 7x7
    (2, 256, 9, 8, 1, 3, 3),
    (11, 36, 1, 12, 0, 2, 2),        # odd group width: scalar path
    (1, 4, 1, 2, 2, 2, 4),
    (64, 24, 5, 3, 0, 4, 4),
    (50, 8192, 1, 8, 2, 7, 1),       # two column blocks, blocks aligned to them
    (97, 16384, 1, 16, 0, 5, 2),     # eight column blocks, 10 blocks: an even split
    (13, 8192, 1, 64, 0, 5, 1),      # four column blocks, 5 blocks: aligned, one extra
]


@pytest.mark.parametrize("shape", SHAPES)
def test_plan_covers_every_element_once(shape):
    batch, channels, inner, groups, dtype, sms, occ = shape
    p = _native.make_plan(batch, channels, inner, groups, dtype, sm_count=sms, ctas_per_sm=occ)
    assert p["group_width"] % p["vec"] == 0
    assert p["vec"] * (4 if dtype == 0 else 2) <= 16
    assert p["threads"] % 32 == 0 and p["threads"] <= 512
    assert p["tile_cols"] * p["tile_rows"] <= p["threads"]
    assert p["blocks"] <= min(p["items"], sms * occ)
    assert p["workspace_bytes"] == p["blocks"] * p["max_segments"] * p["max_local_groups"] * 80
    covered, written, read = simulate(p)
    vec_cols = p["width"] // p["vec"]
    assert len(covered) == batch * vec_cols
    assert set(covered.values()) == {1}
    assert set(read) == set(written) and set(read.values()) == {1}


def test_plan_aligns_blocks_to_column_blocks():
    """A block that crosses a column-block boundary refills its loads and reduces twice; when
    whole blocks per column block cost fewer than a few rows per thread, no block crosses."""
    # x[5461, 8192] bf16 on 148 SMs: two column blocks of 512 vectors, 74 blocks each
    p = _native.make_plan(5461, 8192, 1, 8, 2, sm_count=148, ctas_per_sm=1)
    assert p["col_blocks"] == 2 and p["col_block_blocks"] == 74 and p["col_block_extra"] == 0
    assert p["max_segments"] == 1
    for b in range(p["blocks"]):
        i0, i1 = block_items(p, b)
        assert i0 // p["rows"] == (i1 - 1) // p["rows"]
    sizes = [block_items(p, b)[1] - block_items(p, b)[0] for b in range(p["blocks"])]
    assert max(sizes) - min(sizes) <= 1
    # 64 column blocks of 640 rows on 148 blocks: two or three blocks per column block would
    # give the largest block 320 rows against 277 evenly, more than a refill costs
    p = _native.make_plan(640, 262144, 1, 8, 2, sm_count=148, ctas_per_sm=1)
    assert p["col_blocks"] == 64 and p["col_block_blocks"] == 0


def test_plan_vector_width_follows_group_width():
    assert _native.make_plan(4, 3072, 1, 8, 2)["vec"] == 8
    assert _native.make_plan(4, 768, 1, 64, 2)["vec"] == 4
    assert _native.make_plan(4, 768, 1, 64, 0)["vec"] == 4
    assert _native.make_plan(4, 36, 1, 12, 0)["vec"] == 1
    assert _native.make_plan(4, 16, 49, 8, 2)["vec"] == 2
    assert _native.make_plan(4, 3072, 1, 8, 2, vec=2)["vec"] == 2
    with pytest.raises(_native.KatError):
        _native.make_plan(4, 36, 1, 12, 0, vec=4)


def test_headline_plan_is_balanced():
    """x[128,197,3072] bf16 on 148 SMs: one column block, rows split evenly."""
    p = _native.make_plan(128 * 197, 3072, 1, 8, 2, sm_count=148, ctas_per_sm=1)
    assert p["col_blocks"] == 1 and p["tile_cols"] == 384 and p["blocks"] == 148
    sizes = {block_items(p, b)[1] - block_items(p, b)[0] for b in range(p["blocks"])}
    assert max(sizes) - min(sizes) <= 1


def _divider(d):
    """The multiply-shift constants the library derives for an invariant divisor d
    (Granlund-Montgomery round-up method, N = 64)."""
    l = 0
    while l < 64 and (1 << l) < d:
        l += 1
    m = ((1 << 64) * ((1 << l) - d)) // d + 1
    return m, min(l, 1), max(l - 1, 0)


@pytest.mark.parametrize("d", [1, 2, 3, 7, 48, 197, 25088, 25216, 100352, (1 << 31) - 1,
                               (1 << 40) + 3, (1 << 63)])
def test_invariant_division_formula(d):
    import random

    m, s1, s2 = _divider(d)
    rng = random.Random(d)
    ns = [0, 1, d - 1, d, d + 1, 2 * d - 1, (1 << 63) - 1, (1 << 64) - 1]
    ns += [rng.randrange(0, 1 << 64) for _ in range(200)] + [rng.randrange(0, 1 << 40) for _ in range(200)]
    for n in ns:
        t = (m * n) >> 64
        q = (t + ((n - t) >> s1)) >> s2
        assert q == n // d, (n, d)
