"""Host-side restatement of the fused GEMM's work decomposition (csrc/kat_gemm.cu), checked on
the CPU for the shapes the tests and the KAN block use:

  - the choice between one CTA per 128 x 256 tile and a CTA pair per 256 x 256 tile (pairs only
    when they take no more waves of tiles over the resident CTAs);
  - every CTA (pair) slot takes one contiguous run of the column-block-major tile order, and the
    runs partition the tiles;
  - inside a tile the epilogue warps (8 or 16, warp w reading TMEM lane quadrant w % 4) cover
    the 128 x 256 accumulator exactly once in 32 x 32 chunks;
  - every TMA x coordinate is a multiple of 8 bf16 elements (16 bytes), every box stays inside
    the 16-byte-aligned row pitch, and each mode's shared memory fits the 227 KB limit."""

import itertools

import pytest

BM, BN, BK, CHUNK = 128, 256, 64, 32
SMS, PAIRS = 148, 74
EPI_WARPS = {"plain": 8, "fwd": 8, "bwd": 16}
STAGES = {("plain", 1): 4, ("plain", 2): 6, ("fwd", 1): 4, ("fwd", 2): 6, ("bwd", 1): 3,
          ("bwd", 2): 4}
OUTS = {"plain": 1, "fwd": 2, "bwd": 1}
H_TILES = {"plain": 0, "fwd": 0, "bwd": 1}


def ceil_div(a, b):
    return -(-a // b)


def pairing(m, n):
    t1 = ceil_div(m, BM) * (n // BN)
    t2 = ceil_div(m, 2 * BM) * (n // BN)
    return 2 if ceil_div(t2, PAIRS) <= ceil_div(t1, SMS) else 1


def slots_and_tiles(m, n, pair):
    m_tiles = ceil_div(m, BM * pair)
    tiles = m_tiles * (n // BN)
    cap = PAIRS if pair == 2 else SMS
    return min(cap, tiles), m_tiles, tiles


def smem_bytes(mode, pair):
    a = BM * BK * 2
    b = (BN // pair) * BK * 2
    tile = 32 * CHUNK * 2
    return (1024 + STAGES[(mode, pair)] * (a + b)
            + EPI_WARPS[mode] * (OUTS[mode] + H_TILES[mode]) * tile + 512)


SHAPES = [(128 * 197, 3072, 768), (128, 256, 64), (1, 256, 64), (127, 512, 128), (129, 256, 192),
          (1000, 768, 256), (300, 3072, 768), (333, 3072, 768), (2 * 197, 3072, 768),
          (16 * 197, 512, 128)]


def test_pairing_rule_at_the_vit_shape():
    # 2364 single tiles over 148 SMs: 16 waves; 1188 pair tiles over 74 pairs: 17 waves
    assert pairing(128 * 197, 3072) == 1
    assert pairing(1000, 768) == 2 and pairing(128, 256) == 2


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_tile_runs_partition_the_tiles(m, n, k):
    for pair in (1, 2):
        slots, m_tiles, tiles = slots_and_tiles(m, n, pair)
        seen = []
        for slot in range(slots):
            begin, end = slot * tiles // slots, (slot + 1) * tiles // slots
            seen.extend(range(begin, end))
            assert end - begin in (tiles // slots, ceil_div(tiles, slots))
        assert seen == list(range(tiles))
        # column-block-major: tile -> (row block, column block) is a bijection
        origins = {((t % m_tiles), (t // m_tiles)) for t in range(tiles)}
        assert len(origins) == tiles
        assert all(mb < m_tiles and nb < n // BN for mb, nb in origins)


@pytest.mark.parametrize("mode", ["plain", "fwd", "bwd"])
def test_epilogue_warps_cover_the_tile_once(mode):
    warps = EPI_WARPS[mode]
    slice_cols = BN // (warps // 4)
    covered = {}
    for ew in range(warps):
        warp = ew + 2
        quad, sl = warp & 3, ew >> 2
        for c in range(slice_cols // CHUNK):
            for r, col in itertools.product(range(quad * 32, quad * 32 + 32),
                                            range(sl * slice_cols + c * CHUNK,
                                                  sl * slice_cols + (c + 1) * CHUNK)):
                assert (r, col) not in covered
                covered[(r, col)] = ew
    assert len(covered) == BM * BN
    quads = [((ew + 2) & 3) for ew in range(warps)]
    assert all(quads.count(q) == warps // 4 for q in range(4))


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_tma_coordinates_are_16_byte_aligned(m, n, k):
    for pair in (1, 2):
        _, m_tiles, tiles = slots_and_tiles(m, n, pair)
        for t in range(tiles):
            nb = t // m_tiles
            for rank in range(pair):
                b_row0 = nb * BN + rank * (BN // pair)
                assert b_row0 + BN // pair <= n                # B rows of this CTA exist
                for kb in range(k // BK):
                    assert (kb * BK * 2) % 16 == 0 and kb * BK + BK <= k
            for c in range(BN // CHUNK):
                n0 = nb * BN + c * CHUNK
                assert (n0 * 2) % 16 == 0 and n0 + CHUNK <= n  # output / h boxes
        assert (k * 2) % 16 == 0 and (n * 2) % 16 == 0       # row pitches


@pytest.mark.parametrize("mode,pair", list(STAGES))
def test_shared_memory_fits(mode, pair):
    assert smem_bytes(mode, pair) <= 227 * 1024
