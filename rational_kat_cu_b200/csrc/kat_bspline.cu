// B-spline basis (Cox-de Boor) forward and backward for sm_100a: the basis evaluation of
// efficient-KAN layers that the reference fuses in rational_kat_cu/bspline_basis.py.
//
// Work split: a block of 256 threads takes tiles of 8 R batch rows x 32 features (warp w = rows
// w R .. w R + R - 1, lane = feature; R = 4 or 2 for the cubic layers of grid 5 and 8, whose
// knot count is compiled in, 1 otherwise), walking the tiles of one 32-feature column before
// the next, so it keeps those 32 features' knots in shared memory together with every clamped
// knot difference the recursion divides by, max(t_{j+k} - t_j, 1e-8), and its correctly rounded
// reciprocal (per feature, level k and index j).
//
// Per element, instead of running the recursion over every knot interval (the reference
// evaluates all n_knots - 1 indicators and every level in full), a thread finds the one
// interval t_i <= x < t_{i+1} by binary search and evaluates only the triangle of values that
// can be non-zero there (k + 1 values at level k), each term in the reference's operation order
// — ((x - t_j) / max(t_{j+k} - t_j, 1e-8)) times the lower-order value, the two terms added, no
// fused multiply-add between them — so the non-zero values match the full recursion bit for
// bit and every other basis value is zero, as there.  Each division a / b is evaluated as
// Markstein's FMA-corrected product with the tabulated reciprocal y = RN(1/b):
// q0 = RN(a y), r = a - b q0 (exact, one FMA), q = RN(q0 + r y), which is the correctly
// rounded quotient RN(a / b) (P. Markstein, "Computation of elementary functions on the IBM
// RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990) — the IEEE division result at
// three FP32 operations.  The backward takes the derivative from the order K - 1 values with
// the B-spline identity dB^K_j/dx = K (B^{K-1}_j / d^K_j - B^{K-1}_{j+1} / d^K_{j+1}) (d the
// clamped knot differences), which equals the derivative autograd takes through the recursion
// up to rounding, at the cost of the forward recursion to order K - 1.  Outputs (forward) and
// incoming gradients (backward) go through shared memory so each row of a tile moves as one
// contiguous, coalesced range.
//
// Knots must be non-decreasing along each feature (KANLinear's grid and update_grid produce
// such grids).  A non-finite x gives NaN in every basis value, as the reference's full
// recursion does (its 0 * inf terms).

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>

#include "kat_bspline.h"
#include "kat_rational.h"

namespace {

constexpr int kTileCols = 32;   // features per tile (one warp)
constexpr int kWarps = 8;       // warps per block; warp w takes rows w R .. w R + R - 1 of a tile
constexpr int kBsThreads = kTileCols * kWarps;
// Rows per warp and tile (R): the knot counts of the default cubic layers (grid 5 and 8: 12 and
// 15 knots) are compiled in and take R = 4 or 2 rows per warp, so a warp's loop, column and
// copy bookkeeping is paid once per R elements per lane and its R x loads are in flight
// together; any other order or knot count runs with the knot count at run time and 1 row per
// warp.  R = 4 where four blocks still fit in an SM's shared memory, else 2 (x[16384,1024]
// fp32 on one B200, forward / backward: grid 5 at R = 4 154 / 138 us, at R = 2 160 / 147;
// grid 8, 61.5 KB per block at R = 4, 197 / 158 us there and 177 / 161 at R = 2; R = 8 slower
// for both; 226 / 212 and 223 / 203 us with one row per warp and the knot count at run time).
constexpr size_t kFourBlocksSmem = 56 * 1024;
constexpr int kMaxOrder = 5;
constexpr int kMaxKnots = 64;
constexpr float kEps = 1e-8f;

// RN(a / b) from y = RN(1 / b) (Markstein's correction step).
__device__ __forceinline__ float div_by(float a, float b, float y) {
  const float q0 = __fmul_rn(a, y);
  const float r = __fmaf_rn(-q0, b, a);
  return __fmaf_rn(r, y, q0);
}

// Shared-memory layout of one column of tiles, feature-minor ([index][32 features]): lane c
// reads word index * 32 + c, in its own bank whatever index it needs, so the data-dependent
// span lookups never conflict.  The tables are padded by kOrder entries so that every index a
// span needs is in range without clamping:
//   knots  [n_knots + 2 kOrder][32]   row j + kOrder holds t_{clamp(j, 0, n - 1)}
//   recip  [kOrder][n_knots + kOrder][32]   row (k - 1, j + kOrder): 1 / max(t_{j+k} - t_j, eps)
//   diff   [kOrder][n_knots + kOrder][32]   row (k - 1, j + kOrder): max(t_{j+k} - t_j, eps)
// (recip and diff are 0 / 1 where j < 0 or j + k > n - 1: never read by a valid term).
struct Smem {
  float* knots;
  float* recip;
  float* diff;
  float* slab;    // [8 warps][R rows][32 * n_basis]
};

size_t smem_bytes(int n_knots, int order, int rows_per_warp) {
  const int nb = n_knots - 1 - order;
  return sizeof(float) * kTileCols *
         (size_t(n_knots + 2 * order) + 2 * size_t(order) * (n_knots + order) +
          size_t(kWarps) * rows_per_warp * nb);
}

template <int kOrder>
__host__ __device__ constexpr int table_rows(int n_knots) {
  return n_knots + kOrder;
}

template <int kOrder>
__device__ __forceinline__ Smem carve(float* smem, int n_knots) {
  const int kr = n_knots + 2 * kOrder, tr = table_rows<kOrder>(n_knots);
  Smem sm;
  sm.knots = smem;
  sm.recip = sm.knots + kTileCols * kr;
  sm.diff = sm.recip + kTileCols * kOrder * tr;
  sm.slab = sm.diff + kTileCols * kOrder * tr;
  return sm;
}

// Load the knots of features c0 .. c0 + 31 and tabulate the clamped differences and their
// correctly rounded reciprocals.
template <int kOrder>
__device__ __forceinline__ void load_column(const Smem& sm, const float* __restrict__ grid,
                                            int64_t features, int n_knots, int64_t c0) {
  const int ncols = int(min(int64_t(kTileCols), features - c0));
  const int kr = n_knots + 2 * kOrder, tr = table_rows<kOrder>(n_knots);
  for (int q = threadIdx.x; q < kTileCols * kr; q += kBsThreads) {
    const int c = q % kTileCols, row = q / kTileCols;
    const int j = min(max(row - kOrder, 0), n_knots - 1);
    sm.knots[q] = c < ncols ? grid[(c0 + c) * n_knots + j] : 0.0f;
  }
  __syncthreads();
  const float* t = sm.knots + kTileCols * kOrder;  // t_j at t[j * 32 + c]
  for (int q = threadIdx.x; q < kTileCols * kOrder * tr; q += kBsThreads) {
    const int c = q % kTileCols, kj = q / kTileCols;
    const int k = kj / tr + 1, j = kj - (k - 1) * tr - kOrder;
    float y = 0.0f, d = 1.0f;
    if (j >= 0 && j + k < n_knots) {
      d = fmaxf(__fsub_rn(t[(j + k) * kTileCols + c], t[j * kTileCols + c]), kEps);
      y = __frcp_rn(d);
    }
    sm.recip[q] = y;
    sm.diff[q] = d;
  }
  __syncthreads();
}

// Largest i in [0, n - 2] with t_i <= x, for t_0 <= x < t_{n-1} (non-decreasing t), by binary
// search over the bits of i (a fixed number of steps, no data-dependent branches); knot t_j of
// this lane's feature is t[j * 32].
__host__ __device__ constexpr int pow2_floor(int v) {
  int p = 1;
  while (p * 2 <= v) p *= 2;
  return p;
}
template <int kKnots>   // the knot count when compiled in (> 0), else n at run time
__device__ __forceinline__ int find_span(const float* t, int n, float x) {
  int i = 0;
  const int top = kKnots > 0 ? pow2_floor(kKnots - 2) : 1 << (31 - __clz(n - 2));
  for (int step = top; step > 0; step >>= 1) {
    const int c = i + step;
    if (c <= n - 2 && t[c * kTileCols] <= x) i = c;
  }
  return i;
}

// Everything the triangle of span i reads, moved from shared memory to registers once:
// xl[q] = x - t_{i-kOrder+1+q}, xr[q] = t_{i+1+q} - x (q = 0 .. kOrder - 1), and per level k the
// reciprocals and clamped differences of j = i - k + 1 .. i (rw / dw[k - 1][j - (i - k + 1)]).
// kt points at this lane's padded knots (row j + kOrder = t_j), rc / df at its padded tables.
template <int kOrder>
__device__ __forceinline__ void load_span(const float* kt, const float* rc, const float* df,
                                          int n, int i, float x, float (&xl)[kOrder],
                                          float (&xr)[kOrder], float (&rw)[kOrder][kOrder],
                                          float (&dw)[kOrder][kOrder]) {
  const int tr = table_rows<kOrder>(n);
#pragma unroll
  for (int q = 0; q < kOrder; ++q) {
    xl[q] = __fsub_rn(x, kt[(i + 1 + q) * kTileCols]);               // t_{i-kOrder+1+q}
    xr[q] = __fsub_rn(kt[(i + 1 + q + kOrder) * kTileCols], x);      // t_{i+1+q}
  }
#pragma unroll
  for (int k = 1; k <= kOrder; ++k) {
#pragma unroll
    for (int m = 0; m < k; ++m) {
      const int row = (k - 1) * tr + (i - k + 1 + m + kOrder);
      rw[k - 1][m] = rc[row * kTileCols];
      dw[k - 1][m] = df[row * kTileCols];
    }
  }
}

// Basis values of order kLevels (<= kOrder) that can be non-zero at x in span i:
// b[m] = B^kLevels_{i-kLevels+m} for m = 0..kLevels (entries whose index is outside
// [0, n - 2 - kLevels] are left 0).  Each term is ((numerator / clamped difference) x the lower
// order value), the two terms added without a fused multiply-add, as the reference's recursion.
// The windows are those load_span<kOrder> filled.
template <int kOrder, int kLevels>
__device__ __forceinline__ void span_basis(const float (&xl)[kOrder], const float (&xr)[kOrder],
                                           const float (&rw)[kOrder][kOrder],
                                           const float (&dw)[kOrder][kOrder], int n, int i,
                                           float (&b)[kMaxOrder + 1]) {
  float prev[kMaxOrder + 1];
  prev[0] = 1.0f;
#pragma unroll
  for (int k = 1; k <= kLevels; ++k) {
#pragma unroll
    for (int m = 0; m <= k; ++m) {
      const int j = i - k + m;
      float v = 0.0f;
      if (j >= 0 && j <= n - 2 - k) {
        // left term: (x - t_j) / max(t_{j+k} - t_j, eps) * B^{k-1}_j   (prev index m - 1)
        float left = 0.0f;
        if (m >= 1)
          left = __fmul_rn(div_by(xl[kOrder - 1 - k + m], dw[k - 1][m - 1], rw[k - 1][m - 1]),
                           prev[m - 1]);
        // right term: (t_{j+k+1} - x) / max(t_{j+k+1} - t_{j+1}, eps) * B^{k-1}_{j+1}   (m)
        float right = 0.0f;
        if (m <= k - 1)
          right = __fmul_rn(div_by(xr[m], dw[k - 1][m], rw[k - 1][m]), prev[m]);
        v = __fadd_rn(left, right);
      }
      b[m] = v;
    }
#pragma unroll
    for (int m = 0; m <= k; ++m) prev[m] = b[m];
  }
  if constexpr (kLevels == 0) b[0] = 1.0f;
}

// One forward element: the basis values of x = v of this lane's feature scattered into its
// zeroed slab row r (n_basis floats): NaN in every value for a non-finite x, the k + 1 values of
// its span inside [t_0, t_{n-1}), nothing (zeros) outside.
template <int kOrder, int kKnots>
__device__ __forceinline__ void fwd_element(const Smem& sm, int lane, int n_knots, int nb, float v,
                                            float* r) {
  const float* t = sm.knots + kOrder * kTileCols + lane;   // t_j at t[j * 32]
  if (!isfinite(v)) {
    for (int j = 0; j < nb; ++j) r[j] = __int_as_float(0x7fc00000);
  } else if (v >= t[0] && v < t[(n_knots - 1) * kTileCols]) {
    const int i = find_span<kKnots>(t, n_knots, v);
    float xl[kOrder], xr[kOrder], rw[kOrder][kOrder], dw[kOrder][kOrder];
    load_span<kOrder>(sm.knots + lane, sm.recip + lane, sm.diff + lane, n_knots, i, v, xl, xr,
                      rw, dw);
    float b[kMaxOrder + 1];
    span_basis<kOrder, kOrder>(xl, xr, rw, dw, n_knots, i, b);
#pragma unroll
    for (int m = 0; m <= kOrder; ++m) {
      const int j = i - kOrder + m;
      if (j >= 0 && j < nb) r[j] = b[m];
    }
  }
}

// 16-byte global -> shared copy that bypasses the registers (completed by cp_async_wait_all).
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
               "l"(gmem_src)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}

// Warp-wide copy of `count` floats between a tile row's slab (16-byte aligned) and global
// memory: 16-byte accesses when the global side is 16-byte aligned (towards shared memory as
// cp.async copies, all in flight until the caller's cp_async_wait_all), else 4-byte ones.
template <bool kToGlobal>
__device__ __forceinline__ void warp_copy(float* __restrict__ slab, float* __restrict__ g,
                                          int count, int lane) {
  if ((reinterpret_cast<uintptr_t>(g) & 15) == 0) {
    const int c4 = count >> 2;
    float4* s4 = reinterpret_cast<float4*>(slab);
    float4* g4 = reinterpret_cast<float4*>(g);
    for (int q = lane; q < c4; q += 32) {
      if constexpr (kToGlobal) g4[q] = s4[q]; else cp_async16(s4 + q, g4 + q);
    }
    for (int q = (c4 << 2) + lane; q < count; q += 32) {
      if constexpr (kToGlobal) g[q] = slab[q]; else slab[q] = __ldg(g + q);
    }
  } else {
    for (int q = lane; q < count; q += 32) {
      if constexpr (kToGlobal) g[q] = slab[q]; else slab[q] = __ldg(g + q);
    }
  }
}

// Contiguous range of one tile row: features c0 .. c0 + ncols - 1 of batch row `row`.
__device__ __forceinline__ int64_t row_offset(int64_t row, int64_t features, int64_t c0, int nb) {
  return (row * features + c0) * nb;
}

// Tiles are numbered column-major (all row tiles of feature column 0, then column 1, ...);
// block b takes the contiguous tile range [b * q + min(b, r), ...).
__device__ __forceinline__ void block_tiles(int64_t n_tiles, int64_t& t0, int64_t& t1) {
  const int64_t q = n_tiles / gridDim.x, r = n_tiles % gridDim.x, b = blockIdx.x;
  t0 = b * q + min(b, r);
  t1 = t0 + q + (b < r ? 1 : 0);
}

// Tiles of kWarps R rows x 32 features; warp w owns rows w R .. w R + R - 1 of a tile.
template <int kOrder, int kKnots, int kR>
__global__ void __launch_bounds__(kBsThreads)
kat_bspline_fwd_kernel(const float* __restrict__ x, const float* __restrict__ grid,
                       float* __restrict__ out, int64_t batch, int64_t features, int knots_arg) {
  extern __shared__ __align__(16) float smem[];
  constexpr int kTR = kWarps * kR;
  const int n_knots = kKnots > 0 ? kKnots : knots_arg;
  const int nb = n_knots - 1 - kOrder;
  const int row_floats = kTileCols * nb;   // one slab row: 32 features x n_basis
  const Smem sm = carve<kOrder>(smem, n_knots);
  const int64_t row_tiles = (batch + kTR - 1) / kTR;
  const int64_t col_tiles = (features + kTileCols - 1) / kTileCols;
  int64_t t0, t1;
  block_tiles(row_tiles * col_tiles, t0, t1);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  float* const swarp = sm.slab + w * (kR * row_floats);
  int64_t loaded = -1;
  // (column tile, row tile) of tile t0, then advanced one tile at a time (no division per tile)
  int64_t ct = t0 / row_tiles, rt = t0 - (t0 / row_tiles) * row_tiles;
  for (int64_t tile = t0; tile < t1; ++tile) {
    const int64_t c0 = ct * kTileCols, row0 = rt * kTR + w * kR;
    const int ncols = int(min(int64_t(kTileCols), features - c0));
    if (ct != loaded) {
      __syncthreads();   // the previous column's tables are no longer read
      load_column<kOrder>(sm, grid, features, n_knots, c0);
      loaded = ct;
    }
    // the warp's R x values, loaded before any is used
    float v[kR];
#pragma unroll
    for (int r = 0; r < kR; ++r)
      v[r] = (row0 + r < batch && lane < ncols) ? x[(row0 + r) * features + c0 + lane] : 0.0f;
    {
      float4* s4 = reinterpret_cast<float4*>(swarp);   // R x 32 x nb floats: a multiple of 4
      for (int q = lane; q < (kR * row_floats) >> 2; q += 32) s4[q] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    __syncwarp();
#pragma unroll
    for (int r = 0; r < kR; ++r)
      if (row0 + r < batch && lane < ncols)
        fwd_element<kOrder, kKnots>(sm, lane, n_knots, nb, v[r], swarp + r * row_floats + lane * nb);
    __syncwarp();
#pragma unroll
    for (int r = 0; r < kR; ++r) {
      if (row0 + r >= batch) continue;
      float* g = out + row_offset(row0 + r, features, c0, nb);
      if (kKnots > 0 && ncols == kTileCols)   // a full tile: a compile-time count
        warp_copy<true>(swarp + r * row_floats, g, kTileCols * (kKnots - 1 - kOrder), lane);
      else
        warp_copy<true>(swarp + r * row_floats, g, ncols * nb, lane);
    }
    __syncwarp();
    if (++rt == row_tiles) { rt = 0; ++ct; }
  }
}

// One backward element: dx for x = v of this lane's feature from its incoming-gradient row r
// (n_basis floats): NaN for a non-finite x, 0 outside [t_0, t_{n-1}).
template <int kOrder, int kKnots>
__device__ __forceinline__ float bwd_element(const Smem& sm, int lane, int n_knots, int nb,
                                             float v, const float* r) {
  const float* t = sm.knots + kOrder * kTileCols + lane;   // t_j at t[j * 32]
  float acc = 0.0f;
  if (!isfinite(v)) {
    acc = __int_as_float(0x7fc00000);
  } else if (v >= t[0] && v < t[(n_knots - 1) * kTileCols]) {
    const int i = find_span<kKnots>(t, n_knots, v);
    float xl[kOrder], xr[kOrder], rw[kOrder][kOrder], dw[kOrder][kOrder];
    load_span<kOrder>(sm.knots + lane, sm.recip + lane, sm.diff + lane, n_knots, i, v, xl, xr,
                      rw, dw);
    // dB^K_j / dx = K (B^{K-1}_j / d_j - B^{K-1}_{j+1} / d_{j+1}), d_j = max(t_{j+K} - t_j,
    // eps): the derivative autograd takes through the recursion, from the order K - 1 values
    // (b[m'] = B^{K-1}_{i-K+1+m'}) and the level-K reciprocals.
    float b[kMaxOrder + 1];
    span_basis<kOrder, kOrder - 1>(xl, xr, rw, dw, n_knots, i, b);
#pragma unroll
    for (int m = 0; m <= kOrder; ++m) {
      const int j = i - kOrder + m;
      if (j >= 0 && j < nb) {
        const float left = m >= 1 ? __fmul_rn(b[m - 1], rw[kOrder - 1][m - 1]) : 0.0f;
        const float right = m <= kOrder - 1 ? __fmul_rn(b[m], rw[kOrder - 1][m]) : 0.0f;
        const float d = __fmul_rn(float(kOrder), __fsub_rn(left, right));
        acc = __fadd_rn(acc, __fmul_rn(r[j], d));
      }
    }
  }
  return acc;
}

template <int kOrder, int kKnots, int kR>
__global__ void __launch_bounds__(kBsThreads)
kat_bspline_bwd_kernel(const float* __restrict__ x, const float* __restrict__ grid,
                       const float* __restrict__ gb, float* __restrict__ gx, int64_t batch,
                       int64_t features, int knots_arg) {
  extern __shared__ __align__(16) float smem[];
  constexpr int kTR = kWarps * kR;
  const int n_knots = kKnots > 0 ? kKnots : knots_arg;
  const int nb = n_knots - 1 - kOrder;
  const int row_floats = kTileCols * nb;
  const Smem sm = carve<kOrder>(smem, n_knots);
  const int64_t row_tiles = (batch + kTR - 1) / kTR;
  const int64_t col_tiles = (features + kTileCols - 1) / kTileCols;
  int64_t t0, t1;
  block_tiles(row_tiles * col_tiles, t0, t1);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  float* const swarp = sm.slab + w * (kR * row_floats);
  int64_t loaded = -1;
  // (column tile, row tile) of tile t0, then advanced one tile at a time (no division per tile)
  int64_t ct = t0 / row_tiles, rt = t0 - (t0 / row_tiles) * row_tiles;
  for (int64_t tile = t0; tile < t1; ++tile) {
    const int64_t c0 = ct * kTileCols, row0 = rt * kTR + w * kR;
    const int ncols = int(min(int64_t(kTileCols), features - c0));
    if (ct != loaded) {
      __syncthreads();
      load_column<kOrder>(sm, grid, features, n_knots, c0);
      loaded = ct;
    }
    // with several rows, the warp's x loads are issued before the incoming-gradient copies
    float v[kR];
    auto load_x = [&]() {
#pragma unroll
      for (int r = 0; r < kR; ++r)
        v[r] = (row0 + r < batch && lane < ncols) ? x[(row0 + r) * features + c0 + lane] : 0.0f;
    };
    if constexpr (kR > 1) load_x();
#pragma unroll
    for (int r = 0; r < kR; ++r) {
      if (row0 + r >= batch) continue;
      float* g = const_cast<float*>(gb) + row_offset(row0 + r, features, c0, nb);
      if (kKnots > 0 && ncols == kTileCols)   // a full tile: a compile-time count
        warp_copy<false>(swarp + r * row_floats, g, kTileCols * (kKnots - 1 - kOrder), lane);
      else
        warp_copy<false>(swarp + r * row_floats, g, ncols * nb, lane);
    }
    cp_async_wait_all();
    __syncwarp();
    if constexpr (kR == 1) load_x();
#pragma unroll
    for (int r = 0; r < kR; ++r)
      if (row0 + r < batch && lane < ncols)
        gx[(row0 + r) * features + c0 + lane] =
            bwd_element<kOrder, kKnots>(sm, lane, n_knots, nb, v[r], swarp + r * row_floats + lane * nb);
    __syncwarp();
    if (++rt == row_tiles) { rt = 0; ++ct; }
  }
}

int validate(int64_t batch, int64_t features, int32_t n_knots, int32_t order, int64_t* n) {
  if (batch < 0 || features < 0) return KAT_ERR_BAD_SHAPE;
  if (order < 1 || order > kMaxOrder || n_knots < order + 2 || n_knots > kMaxKnots)
    return KAT_ERR_BAD_SHAPE;
  if (features != 0 && batch > (int64_t(1) << 40) / features) return KAT_ERR_BAD_SHAPE;
  *n = batch * features;
  return KAT_OK;
}

// Grid: as many blocks as fit on the GPU at once, never more than there are tiles.
cudaError_t grid_size(int64_t batch, int64_t features, int tile_rows, const void* fn, size_t smem,
                      unsigned* blocks) {
  int dev = 0, sms = 0, occ = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e == cudaSuccess && smem > 48 * 1024)
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, kBsThreads, smem);
  if (e != cudaSuccess) return e;
  const int64_t tiles = ((batch + tile_rows - 1) / tile_rows) *
                        ((features + kTileCols - 1) / kTileCols);
  *blocks = unsigned(std::max<int64_t>(1, std::min<int64_t>(tiles, int64_t(sms) * std::max(occ, 1))));
  return cudaSuccess;
}

template <int kOrder, int kKnots, int kR>
cudaError_t launch_fwd_k(const float* x, const float* grid, float* out, int64_t batch, int64_t f,
                         int nk, cudaStream_t s) {
  const size_t smem = smem_bytes(nk, kOrder, kR);
  auto kernel = kat_bspline_fwd_kernel<kOrder, kKnots, kR>;
  unsigned blocks = 0;
  const cudaError_t e = grid_size(batch, f, kWarps * kR, (const void*)kernel, smem, &blocks);
  if (e != cudaSuccess) return e;
  kernel<<<blocks, kBsThreads, smem, s>>>(x, grid, out, batch, f, nk);
  return cudaGetLastError();
}

template <int kOrder, int kKnots, int kR>
cudaError_t launch_bwd_k(const float* x, const float* grid, const float* gb, float* gx,
                         int64_t batch, int64_t f, int nk, cudaStream_t s) {
  const size_t smem = smem_bytes(nk, kOrder, kR);
  auto kernel = kat_bspline_bwd_kernel<kOrder, kKnots, kR>;
  unsigned blocks = 0;
  const cudaError_t e = grid_size(batch, f, kWarps * kR, (const void*)kernel, smem, &blocks);
  if (e != cudaSuccess) return e;
  kernel<<<blocks, kBsThreads, smem, s>>>(x, grid, gb, gx, batch, f, nk);
  return cudaGetLastError();
}

// Rows per warp of the compiled-in cubic kernel for `knots` knots (see kFourBlocksSmem).
constexpr int rows_for(int knots) {
  return sizeof(float) * kTileCols *
                     (size_t(knots + 6) + 6 * size_t(knots + 3) +
                      size_t(kWarps) * 4 * (knots - 4)) <= kFourBlocksSmem
             ? 4
             : 2;
}

// Cubic layers with grid 5 or 8 (12 or 15 knots) take the compiled-in kernels; every other
// order and knot count the general ones.
template <int kOrder>
cudaError_t launch_fwd(const float* x, const float* grid, float* out, int64_t batch, int64_t f,
                       int nk, cudaStream_t s) {
  if constexpr (kOrder == 3) {
    if (nk == 12) return launch_fwd_k<3, 12, rows_for(12)>(x, grid, out, batch, f, nk, s);
    if (nk == 15) return launch_fwd_k<3, 15, rows_for(15)>(x, grid, out, batch, f, nk, s);
  }
  return launch_fwd_k<kOrder, 0, 1>(x, grid, out, batch, f, nk, s);
}

template <int kOrder>
cudaError_t launch_bwd(const float* x, const float* grid, const float* gb, float* gx,
                       int64_t batch, int64_t f, int nk, cudaStream_t s) {
  if constexpr (kOrder == 3) {
    if (nk == 12) return launch_bwd_k<3, 12, rows_for(12)>(x, grid, gb, gx, batch, f, nk, s);
    if (nk == 15) return launch_bwd_k<3, 15, rows_for(15)>(x, grid, gb, gx, batch, f, nk, s);
  }
  return launch_bwd_k<kOrder, 0, 1>(x, grid, gb, gx, batch, f, nk, s);
}
static_assert(rows_for(12) == 4 && rows_for(15) == 2, "cubic grid 5 / grid 8 rows per warp");

}  // namespace

extern "C" {

int kat_bspline_basis_fwd(const float* x, const float* grid, float* bases, int64_t batch,
                          int64_t features, int32_t n_knots, int32_t spline_order,
                          void* stream) {
  int64_t n = 0;
  const int st = validate(batch, features, n_knots, spline_order, &n);
  if (st != KAT_OK) return st;
  if (n == 0) return KAT_OK;
  if (x == nullptr || grid == nullptr || bases == nullptr) return KAT_ERR_NULL_POINTER;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  switch (spline_order) {
    case 1: e = launch_fwd<1>(x, grid, bases, batch, features, n_knots, s); break;
    case 2: e = launch_fwd<2>(x, grid, bases, batch, features, n_knots, s); break;
    case 3: e = launch_fwd<3>(x, grid, bases, batch, features, n_knots, s); break;
    case 4: e = launch_fwd<4>(x, grid, bases, batch, features, n_knots, s); break;
    default: e = launch_fwd<5>(x, grid, bases, batch, features, n_knots, s); break;
  }
  return e == cudaSuccess ? KAT_OK : KAT_ERR_CUDA;
}

int kat_bspline_basis_bwd(const float* x, const float* grid, const float* grad_bases,
                          float* grad_x, int64_t batch, int64_t features, int32_t n_knots,
                          int32_t spline_order, void* stream) {
  int64_t n = 0;
  const int st = validate(batch, features, n_knots, spline_order, &n);
  if (st != KAT_OK) return st;
  if (n == 0) return KAT_OK;
  if (x == nullptr || grid == nullptr || grad_bases == nullptr || grad_x == nullptr)
    return KAT_ERR_NULL_POINTER;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  switch (spline_order) {
    case 1: e = launch_bwd<1>(x, grid, grad_bases, grad_x, batch, features, n_knots, s); break;
    case 2: e = launch_bwd<2>(x, grid, grad_bases, grad_x, batch, features, n_knots, s); break;
    case 3: e = launch_bwd<3>(x, grid, grad_bases, grad_x, batch, features, n_knots, s); break;
    case 4: e = launch_bwd<4>(x, grid, grad_bases, grad_x, batch, features, n_knots, s); break;
    default: e = launch_bwd<5>(x, grid, grad_bases, grad_x, batch, features, n_knots, s); break;
  }
  return e == cudaSuccess ? KAT_OK : KAT_ERR_CUDA;
}

}  // extern "C"
