// Host-only check of the launch planner (csrc/kat_plan.h), built by
// tests/test_native_sanitized.py with -fsanitize=address,undefined -fno-sanitize-recover=all
// so that any out-of-bounds access, signed overflow or invalid shift in the planner aborts.
//
// Checked, over a grid of shapes, dtypes, vector widths and device sizes (plus random ones):
//  * make_divider: the multiply-shift quotient equals n / d (the kernels' fast_div, restated
//    here with a 128-bit product) for divisors 1 .. 2^62 and dividends up to 2^63 - 1;
//  * make_plan_impl: every accepted plan covers each row and vector column exactly once, its
//    blocks' item ranges tile [0, items), each block touches at most max_segments column
//    blocks (one when the split is aligned to column blocks, whose blocks then differ by at
//    most one item within a column block), each column block holds at most max_local_groups groups, the partial-sum
//    workspace is exactly blocks x segments x local groups x 10 doubles, and the block size is
//    a multiple of 32 within the cap.
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <random>
#include <vector>

#include "kat_rational.h"

namespace {
#include "kat_plan.h"

int failures = 0;

#define EXPECT(cond, ...)                                 \
  do {                                                    \
    if (!(cond)) {                                        \
      if (failures < 20) {                                \
        fprintf(stderr, "FAIL %s:%d: ", __FILE__, __LINE__); \
        fprintf(stderr, __VA_ARGS__);                     \
        fprintf(stderr, "\n");                            \
      }                                                   \
      ++failures;                                         \
    }                                                     \
  } while (0)

uint64_t host_fast_div(uint64_t n, uint64_t m, int32_t s1, int32_t s2) {
  const uint64_t t = uint64_t(((unsigned __int128)m * n) >> 64);
  return (t + ((n - t) >> s1)) >> s2;
}

void check_divider(std::mt19937_64& rng) {
  std::vector<uint64_t> ds;
  for (uint64_t d = 1; d <= 4096; ++d) ds.push_back(d);
  for (int b = 1; b < 63; ++b) {
    const uint64_t p = uint64_t(1) << b;
    ds.push_back(p - 1);
    ds.push_back(p);
    ds.push_back(p + 1);
  }
  for (int i = 0; i < 2000; ++i) ds.push_back((rng() >> (rng() % 63)) | 1);
  const uint64_t nmax = (uint64_t(1) << 63) - 1;
  for (uint64_t d : ds) {
    if (d == 0 || d > (uint64_t(1) << 62)) continue;
    uint64_t m;
    int32_t s1, s2;
    make_divider(d, &m, &s1, &s2);
    std::vector<uint64_t> ns = {0, 1, d - 1, d, d + 1, 2 * d - 1, 2 * d, nmax, nmax - 1,
                                nmax / d * d, nmax / d * d - 1};
    for (int i = 0; i < 64; ++i) ns.push_back(rng() & nmax);
    for (int i = 0; i < 16; ++i) ns.push_back((rng() % 1000000) * d + (rng() % d));
    for (uint64_t n : ns) {
      if (n > nmax) continue;
      EXPECT(host_fast_div(n, m, s1, s2) == n / d, "fast_div(%llu / %llu)",
             (unsigned long long)n, (unsigned long long)d);
    }
  }
}

void block_range(const Plan& p, int64_t blk, int64_t* i0, int64_t* i1) {
  block_items(p, blk, *i0, *i1);
}

int64_t plans_checked = 0;
int64_t aligned_plans = 0;

void check_plan(int64_t batch, int64_t channels, int64_t inner, int64_t groups, int dtype, int vec,
                int sms, int ctas, int max_cols, int max_threads) {
  Plan p;
  const int st = make_plan_impl(batch, channels, inner, groups, dtype, vec, sms, ctas, &p,
                                max_cols, max_threads);
  if (st != KAT_OK) return;
  ++plans_checked;
  EXPECT(p.rows == batch && p.width == channels * inner, "dims");
  EXPECT(p.vec >= 1 && p.group_width % p.vec == 0 && p.width % p.vec == 0, "vec %d", p.vec);
  if (batch * p.width == 0) return;
  EXPECT(p.threads % 32 == 0 && p.threads >= 32, "threads %d", p.threads);
  EXPECT(int64_t(p.tile_cols) * p.tile_rows <= p.threads, "tile fits the block");
  EXPECT(p.threads <= ((max_threads + 31) / 32) * 32 || p.tile_cols > max_threads, "cap");
  EXPECT(p.tile_rows >= 1 && p.tile_rows <= batch, "tile_rows %d", p.tile_rows);
  EXPECT(int64_t(p.tile_cols) * p.col_blocks >= p.vec_cols, "columns covered");
  EXPECT(int64_t(p.tile_cols) * (p.col_blocks - 1) < p.vec_cols, "no empty column block");
  EXPECT(p.items == p.col_blocks * batch, "items");
  EXPECT(p.blocks >= 1 && p.blocks <= p.items && p.blocks <= kMaxBlocks, "blocks");
  int64_t expect_i0 = 0;
  for (int64_t b = 0; b < p.blocks; ++b) {
    int64_t i0, i1;
    block_range(p, b, &i0, &i1);
    EXPECT(i0 == expect_i0 && i1 > i0, "block %lld range", (long long)b);
    expect_i0 = i1;
    const int64_t cb0 = i0 / p.rows, cb1 = (i1 - 1) / p.rows;
    EXPECT(cb1 - cb0 + 1 <= p.max_segments, "segments %lld > %d", (long long)(cb1 - cb0 + 1),
           p.max_segments);
    uint64_t m;
    int32_t s1, s2;
    make_divider(uint64_t(p.rows), &m, &s1, &s2);
    EXPECT(m == p.rows_m && s1 == p.rows_s1 && s2 == p.rows_s2, "rows divider");
    EXPECT(int64_t(host_fast_div(uint64_t(i0), p.rows_m, p.rows_s1, p.rows_s2)) == cb0, "cb0");
  }
  EXPECT(expect_i0 == p.items, "ranges tile the items");
  if (p.cb_q > 0) {
    // Aligned split: every block inside one column block, sizes within a column block differ
    // by at most one, and the largest block is at most kStraddleRows tile rows above the even
    // split's largest.
    ++aligned_plans;
    EXPECT(p.max_segments == 1, "aligned plan with %d segments", p.max_segments);
    EXPECT(p.cb_q * p.col_blocks + p.cb_r == p.blocks && p.cb_r < p.col_blocks, "aligned counts");
    const int64_t even_max = (p.items + p.blocks - 1) / p.blocks;
    int64_t prev_cb = -1, lo = 0, hi = 0;
    for (int64_t b = 0; b <= p.blocks; ++b) {
      int64_t i0 = 0, i1 = 0, cb = -2;
      if (b < p.blocks) {
        block_range(p, b, &i0, &i1);
        cb = i0 / p.rows;
        EXPECT((i1 - 1) / p.rows == cb, "aligned block %lld crosses a column block", (long long)b);
        EXPECT(i1 - i0 < even_max + int64_t(kStraddleRows) * p.tile_rows, "aligned block size");
      }
      if (cb != prev_cb) {
        if (prev_cb >= 0) EXPECT(hi - lo <= 1, "column block %lld sizes %lld..%lld", (long long)prev_cb, (long long)lo, (long long)hi);
        lo = hi = i1 - i0;
        prev_cb = cb;
      } else {
        lo = i1 - i0 < lo ? i1 - i0 : lo;
        hi = i1 - i0 > hi ? i1 - i0 : hi;
      }
    }
  }
  for (int64_t cb = 0; cb < p.col_blocks; ++cb) {
    const int64_t col0 = cb * p.tile_cols;
    int64_t col_end = col0 + p.tile_cols;
    if (col_end > p.vec_cols) col_end = p.vec_cols;
    const int64_t g0 = col0 / p.vec_group, g1 = (col_end - 1) / p.vec_group;
    EXPECT(g1 - g0 + 1 <= p.max_local_groups, "local groups");
    EXPECT(int64_t(host_fast_div(uint64_t(col0), p.vg_m, p.vg_s1, p.vg_s2)) == g0, "g0");
    if (cb > 4 && cb < p.col_blocks - 4) cb = p.col_blocks - 4;  // ends are enough
  }
  EXPECT(p.workspace_bytes == uint64_t(p.blocks) * uint64_t(p.max_segments) *
                                  uint64_t(p.max_local_groups) * kPlanSums * sizeof(double),
         "workspace");
}

}  // namespace

int main() {
  std::mt19937_64 rng(1234);
  check_divider(rng);
  const int64_t batches[] = {0, 1, 2, 3, 7, 64, 197, 1000, 1576, 25216, (int64_t(1) << 20) + 1,
                             (int64_t(1) << 31) + 5};
  const int64_t channels[] = {1, 2, 3, 12, 36, 64, 256, 768, 3072, 8192, 65536};
  const int64_t inners[] = {0, 1, 2, 7, 49, 3136};
  const int64_t group_opts[] = {1, 2, 3, 4, 8, 12, 16, 64};
  const int dtypes[] = {KAT_DTYPE_F32, KAT_DTYPE_F16, KAT_DTYPE_BF16};
  for (int64_t b : batches)
    for (int64_t c : channels)
      for (int64_t in : inners)
        for (int64_t g : group_opts) {
          if (c % g != 0) continue;
          for (int dt : dtypes)
            for (int vec : {0, 1, 2, 4, 8})
              for (int sms : {1, 148})
                for (int ctas : {1, 2})
                  for (int cols : {128, 512})
                    check_plan(b, c, in, g, dt, vec, sms, ctas, cols, cols == 128 ? 640 : 512);
        }
  for (int i = 0; i < 20000; ++i) {
    const int64_t c = int64_t(1 + rng() % 10000);
    int64_t g = int64_t(1 + rng() % 64);
    while (c % g) --g;
    check_plan(int64_t(rng() % 100000), c, int64_t(1 + rng() % 64), g, int(rng() % 3),
               int(rng() % 2 ? 0 : 1 << (rng() % 4)), int(1 + rng() % 200), int(1 + rng() % 4),
               int(32 * (1 + rng() % 16)), int(32 * (1 + rng() % 20)));
  }
  // Refill estimate behind the cp.async backward's tile width: x[64,256,56,56] fp32 NCHW
  // (64 rows of 200,704 vectors) crosses ~11 column blocks per block at 128 columns and ~3 at
  // 512; x[25216, 3072] bf16 has one column block per block at 128 columns (aligned split).
  {
    Plan narrow, wide, headline;
    EXPECT(make_plan_impl(64, 256, 3136, 8, KAT_DTYPE_F32, 4, 148, 1, &narrow, 128, 512) == KAT_OK &&
               make_plan_impl(64, 256, 3136, 8, KAT_DTYPE_F32, 4, 148, 1, &wide, 512, 512) == KAT_OK,
           "NCHW plans");
    EXPECT(narrow.threads == 512 && wide.threads == 512, "full blocks");
    EXPECT(refill_overhead(narrow) > 0.3 && refill_overhead(wide) < 0.12 &&
               refill_overhead(wide) < refill_overhead(narrow) - 0.02,
           "NCHW refills %f vs %f", refill_overhead(narrow), refill_overhead(wide));
    EXPECT(make_plan_impl(25216, 3072, 1, 8, KAT_DTYPE_BF16, 8, 148, 1, &headline, 128, 512) ==
                   KAT_OK &&
               headline.cb_q > 0 && refill_overhead(headline) == 0.0,
           "headline refills");
  }
  // Invalid requests are refused, not planned.
  Plan p;
  EXPECT(make_plan_impl(-1, 8, 1, 1, KAT_DTYPE_F32, 0, 148, 1, &p) == KAT_ERR_BAD_SHAPE, "neg");
  EXPECT(make_plan_impl(4, 8, 1, 3, KAT_DTYPE_F32, 0, 148, 1, &p) == KAT_ERR_BAD_GROUPS, "G");
  EXPECT(make_plan_impl(int64_t(1) << 40, int64_t(1) << 20, 1, 1, KAT_DTYPE_F32, 0, 148, 1, &p) ==
             KAT_ERR_BAD_SHAPE, "too large");
  EXPECT(make_plan_impl(4, 8, 1, 1, 7, 0, 148, 1, &p) == KAT_ERR_BAD_DTYPE, "dtype");
  EXPECT(make_plan_impl(4, 8, 1, 1, KAT_DTYPE_F32, 3, 148, 1, &p) == KAT_ERR_BAD_SHAPE, "vec");
  if (failures) {
    fprintf(stderr, "%d failures\n", failures);
    return 1;
  }
  EXPECT(aligned_plans > 0 && aligned_plans < plans_checked, "aligned plans %lld of %lld",
         (long long)aligned_plans, (long long)plans_checked);
  printf("ok %lld plans (%lld aligned to column blocks)\n", (long long)plans_checked,
         (long long)aligned_plans);
  return 0;
}
