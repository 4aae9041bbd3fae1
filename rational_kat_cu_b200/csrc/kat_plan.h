// kat_plan.h — launch geometry of the group-rational kernels: plain host C++ (no CUDA), so
// the planner can be built and checked on its own (tests/native/plan_check.cpp compiles it
// under AddressSanitizer and UndefinedBehaviorSanitizer).  Included inside the anonymous
// namespace of kat_rational.cu after kat_rational.h, <stdint.h> and <string.h>.
#pragma once

#ifdef __CUDACC__
#define KAT_PLAN_HD __host__ __device__ __forceinline__
#else
#define KAT_PLAN_HD inline
#endif

constexpr int kPlanSums = 10;      // fp64 partial sums per (block, segment, group): 6 + 4 moments
constexpr int kMaxThreads = 512;  // block size cap
constexpr int64_t kMaxElements = int64_t(1) << 48;
constexpr int64_t kMaxBlocks = int64_t(1) << 14;
// A block whose item range crosses a column-block boundary refills its loads from empty and
// reduces twice: measured on B200 (x[5461, 3072] and x[25216, 3072] bf16 backward, 148 blocks)
// such a block finishes 4.5-5 us after the others, about the time of 6 rows per thread of work
// (the cp.async backward keeps 6 rows per thread in flight).  The planner gives each column
// block whole blocks when that costs less than this many rows per thread.
constexpr int kStraddleRows = 6;

// Launch geometry shared by host and device (a POD copy of kat_rational_plan).
struct Plan {
  int64_t rows;
  int64_t width;
  int64_t group_width;
  int64_t num_groups;
  int64_t vec_cols;    // vectors per row
  int64_t vec_group;   // vectors per group
  int64_t col_blocks;
  int64_t items;
  int64_t blocks;
  int32_t vec;
  int32_t threads;
  int32_t tile_cols;
  int32_t tile_rows;
  int32_t max_segments;
  int32_t max_local_groups;
  uint64_t workspace_bytes;
  int64_t items_q;     // items per block, floor(items / blocks)
  int64_t items_r;     // the first items_r blocks take one more item
  // Split aligned to column blocks (cb_q > 0): the first cb_r column blocks get cb_q + 1
  // blocks and the others cb_q; a column block's rows are split evenly over its blocks
  // (rq_hi / rr_hi: quotient and remainder of rows by cb_q + 1, rq_lo / rr_lo: by cb_q).
  // cb_q == 0: the items are split evenly over all blocks (items_q / items_r).
  int64_t cb_q, cb_r, rq_hi, rr_hi, rq_lo, rr_lo;
  uint64_t rows_m;     // multiply-shift constants for dividing by rows ...
  uint64_t vg_m;       // ... and by vec_group
  int32_t rows_s1, rows_s2, vg_s1, vg_s2;
  int32_t formula;     // KAT_FORMULA_*: how the reduction signs the denominator terms
  int32_t num_stride;  // floats between groups' numerator rows: 6, or 0 for one shared row
};

// Division by an invariant divisor d >= 1 with a multiply and shifts (Granlund and
// Montgomery, "Division by invariant integers using multiplication", PLDI 1994, the
// round-up method of their Figure 4.1 for N = 64): with l = ceil(log2 d),
// m = floor(2^64 (2^l - d) / d) + 1, sh1 = min(l, 1), sh2 = max(l - 1, 0):
//   t = mulhi(m, n);  n / d = (t + ((n - t) >> sh1)) >> sh2   for all 0 <= n < 2^64.
void make_divider(uint64_t d, uint64_t* m, int32_t* s1, int32_t* s2) {
  int l = 0;
  while (l < 64 && (uint64_t(1) << l) < d) ++l;
  const unsigned __int128 two64 = (unsigned __int128)1 << 64;
  const unsigned __int128 num = two64 * (((unsigned __int128)1 << l) - d);
  *m = uint64_t(num / d + 1);
  *s1 = l < 1 ? l : 1;
  *s2 = l - 1 > 0 ? l - 1 : 0;
}

int elem_bytes(int dtype) { return dtype == KAT_DTYPE_F32 ? 4 : 2; }

int validate_dims(int64_t batch, int64_t channels, int64_t inner, int64_t num_groups, int dtype,
                  int64_t* n_elems) {
  if (dtype != KAT_DTYPE_F32 && dtype != KAT_DTYPE_F16 && dtype != KAT_DTYPE_BF16)
    return KAT_ERR_BAD_DTYPE;
  if (batch < 0 || channels < 0 || inner < 0) return KAT_ERR_BAD_SHAPE;
  if (num_groups < 1 || channels % num_groups != 0) return KAT_ERR_BAD_GROUPS;
  if (inner != 0 && channels > kMaxElements / inner) return KAT_ERR_BAD_SHAPE;
  const int64_t width = channels * inner;
  if (width != 0 && batch > kMaxElements / width) return KAT_ERR_BAD_SHAPE;
  *n_elems = batch * width;
  return KAT_OK;
}

int max_vec_for(int dtype) { return 16 / elem_bytes(dtype); }

int make_plan_impl(int64_t batch, int64_t channels, int64_t inner, int64_t num_groups, int dtype,
                   int vec, int sm_count, int ctas_per_sm, Plan* p, int max_cols = kMaxThreads,
                   int max_threads = kMaxThreads) {
  int64_t n = 0;
  int st = validate_dims(batch, channels, inner, num_groups, dtype, &n);
  if (st != KAT_OK) return st;
  if (sm_count < 1 || ctas_per_sm < 1) return KAT_ERR_BAD_SHAPE;
  memset(p, 0, sizeof(*p));
  p->rows = batch;
  p->width = channels * inner;
  p->group_width = (channels / num_groups) * inner;
  p->num_groups = num_groups;
  const int vmax = max_vec_for(dtype);
  if (vec == 0) {
    vec = vmax;
    while (vec > 1 && p->group_width % vec != 0) vec >>= 1;
  } else if (vec < 1 || vec > vmax || (vec & (vec - 1)) != 0 || p->group_width % vec != 0) {
    return KAT_ERR_BAD_SHAPE;
  }
  p->vec = vec;
  p->vec_cols = p->width / vec;
  p->vec_group = p->group_width / vec;
  if (n == 0) {
    p->threads = 32;
    p->tile_cols = 1;
    p->tile_rows = 1;
    return KAT_OK;
  }
  if (p->vec_cols <= max_cols) {
    p->tile_cols = int32_t(p->vec_cols);
  } else {
    const int64_t ncb = (p->vec_cols + max_cols - 1) / max_cols;
    int64_t tcols = (p->vec_cols + ncb - 1) / ncb;
    tcols = (tcols + 31) / 32 * 32;
    if (tcols > max_cols) tcols = max_cols;
    p->tile_cols = int32_t(tcols);
  }
  {
    int64_t tr = max_threads / p->tile_cols;
    if (tr > batch) tr = batch;
    if (tr < 1) tr = 1;
    p->tile_rows = int32_t(tr);
  }
  const int64_t used = int64_t(p->tile_cols) * p->tile_rows;
  p->threads = int32_t((used + 31) / 32 * 32);
  p->col_blocks = (p->vec_cols + p->tile_cols - 1) / p->tile_cols;
  p->items = p->col_blocks * batch;
  int64_t blocks = int64_t(sm_count) * ctas_per_sm;
  if (blocks > kMaxBlocks) blocks = kMaxBlocks;
  if (blocks > p->items) blocks = p->items;
  p->blocks = blocks;
  const int64_t per_block = (p->items + blocks - 1) / blocks;
  int64_t segs = (per_block - 1) / batch + 2;
  if (segs > p->col_blocks) segs = p->col_blocks;
  if (p->col_blocks > 1 && blocks >= p->col_blocks) {
    const int64_t q = blocks / p->col_blocks;
    const int64_t aligned = (batch + q - 1) / q;   // largest block of a column block with q
    if (batch > q && aligned - per_block < int64_t(kStraddleRows) * p->tile_rows) {
      p->cb_q = q;
      p->cb_r = blocks % p->col_blocks;
      p->rq_hi = batch / (q + 1);
      p->rr_hi = batch % (q + 1);
      p->rq_lo = batch / q;
      p->rr_lo = batch % q;
      segs = 1;
    }
  }
  p->max_segments = int32_t(segs);
  int64_t lg = (int64_t(p->tile_cols) - 1) / p->vec_group + 2;
  if (lg > num_groups) lg = num_groups;
  p->max_local_groups = int32_t(lg);
  p->workspace_bytes = uint64_t(blocks) * uint64_t(segs) * uint64_t(lg) * kPlanSums * sizeof(double);
  p->items_q = p->items / blocks;
  p->items_r = p->items % blocks;
  make_divider(uint64_t(batch), &p->rows_m, &p->rows_s1, &p->rows_s2);
  make_divider(uint64_t(p->vec_group), &p->vg_m, &p->vg_s1, &p->vg_s2);
  return KAT_OK;
}

// Extra load-ring refills a plan costs, as a fraction of a thread's rows: a block refills its
// ring at every column block it enters after the first (kStraddleRows rows of work each), and
// works through per_block / tile_rows rows per thread.  Short, wide problems (few rows, many
// column blocks: x[64,256,56,56] NCHW is 64 rows of 200,704 vectors) pay several refills per
// block with narrow tiles; the cp.async backward's planner compares tile widths with it.
inline double refill_overhead(const Plan& p) {
  if (p.items == 0 || p.blocks == 0 || p.rows == 0) return 0.0;
  const double per_block = double(p.items) / double(p.blocks);
  const double segments = p.cb_q > 0 ? 1.0 : per_block / double(p.rows) + 1.0;
  const double rows_per_thread = per_block / double(p.tile_rows);
  return (segments - 1.0) * kStraddleRows / rows_per_thread;
}

// Item range [i0, i1) of block `blk`: an even split of all items (sizes differ by at most
// one), or, when the plan aligns blocks to column blocks, an even split of one column block's
// rows.  Every block gets at least one item.
KAT_PLAN_HD void block_items(const Plan& p, int64_t blk, int64_t& i0, int64_t& i1) {
  if (p.cb_q == 0) {
    i0 = blk * p.items_q + (blk < p.items_r ? blk : p.items_r);
    i1 = i0 + p.items_q + (blk < p.items_r ? 1 : 0);
    return;
  }
  const int64_t hi = p.cb_q + 1;
  const int64_t first_lo = p.cb_r * hi;   // first block of the column blocks with cb_q blocks
  int64_t cb, k, rq, rr;
  if (blk < first_lo) {
    cb = blk / hi;
    k = blk - cb * hi;
    rq = p.rq_hi;
    rr = p.rr_hi;
  } else {
    const int64_t j = (blk - first_lo) / p.cb_q;
    cb = p.cb_r + j;
    k = blk - first_lo - j * p.cb_q;
    rq = p.rq_lo;
    rr = p.rr_lo;
  }
  i0 = cb * p.rows + k * rq + (k < rr ? k : rr);
  i1 = i0 + rq + (k < rr ? 1 : 0);
}
