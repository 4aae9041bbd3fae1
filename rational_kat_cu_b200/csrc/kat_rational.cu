// kat_rational.cu — sm_100a kernels and C ABI for KAT's group-rational activation.
//
// Formula (kat_rational/kat_1dgroup_torch.py:27-78 of the reference):
//   y = P(x) / Q(x),  P = sum_{k=0..5} a_k x^k,  Q = 1 + sum_{i=1..4} |b_i| x^i
// evaluated per channel group.  Gradients are those torch autograd derives for
// that formula (abs backward uses sgn, so sgn(0) = 0):
//   dx      = go * (P' Q - P Q') / Q^2
//   d a_k   = sum go x^k / Q
//   d b_i   = sgn(b_i) * sum -go P x^i / Q^2
//
// Work decomposition (both kernels).  A contiguous tensor is viewed as
// [rows, width] with width = channels * inner; a group is a run of
// group_width = (channels / G) * inner consecutive columns, so channels-last
// ([B*L, C], inner = 1) and NCHW ([B, C*H*W]) share one kernel family.
// Columns are read as vectors of `vec` elements (16 bytes when the shape and
// pointers allow).  A block is a tile of tile_cols vector columns x tile_rows
// rows; the row is split into col_blocks column blocks, and the "items"
// (column block, row) are divided evenly over a persistent grid of
// blocks = SMs x occupancy, each block taking one contiguous item range.
// Inside a range a thread keeps one fixed vector column, so its group — and
// its coefficients and gradient accumulators — stay in registers.
//
// Backward reduction (no floating-point atomics, fixed order): per-thread fp32
// sums -> per-block fp64 sums per (segment, group) written to the workspace ->
// a second kernel that adds, for every group, the workspace entries of all
// blocks in block order, in fp64.  The decomposition depends only on the
// shape, dtype, vector width and the device's SM count and occupancy, so
// results are bit-identical from run to run on the same GPU model.
//
// Arithmetic is fp32.  Pairs of elements go through the sm_100 paired-fp32
// instructions (__ffma2_rn / __fmul2_rn), halving instruction issue.
// Reciprocals use the PTX rcp.approx instruction (max error 1 ulp); the fp32
// backward adds one Newton-Raphson step, and the fp32 forward uses the
// correctly rounded division __fdiv_rn.

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <map>
#include <type_traits>
#include <mutex>
#include <tuple>

#include "kat_rational.h"

namespace {

#include "kat_math.cuh"

#include "kat_plan.h"

static_assert(kPlanSums == kAcc, "workspace slots per group: the 10 gradient moments");
constexpr int kReduceThreads = kAcc * 32;

__device__ int g_kat_status;  // sticky device status (0 = ok), read by kat_rational_device_status

// Bounds-checked build (-DKAT_DEBUG_BOUNDS=1: libkat_rational_debug.so).  Every global access
// of the activation kernels, every workspace slot and the plan's segment / group invariants
// are checked before the access is made: a violation sets KAT_DEVICE_BOUNDS in the sticky
// status word and the access is skipped — never a trap, so a shared GPU is never faulted.
// In the release build the checks compile away.
constexpr int kStatusBounds = KAT_DEVICE_BOUNDS;
#ifndef KAT_DEBUG_BOUNDS
#define KAT_DEBUG_BOUNDS 0
#endif
__device__ __forceinline__ bool kat_check(bool ok) {
#if KAT_DEBUG_BOUNDS
  if (!ok) atomicExch(&g_kat_status, kStatusBounds);
  return ok;
#else
  (void)ok;
  return true;
#endif
}
// [ptr, ptr + n) inside [base, base + count) (element units).
template <typename T>
__device__ __forceinline__ bool in_bounds(const T* base, int64_t count, const T* ptr,
                                          int64_t n = 1) {
#if KAT_DEBUG_BOUNDS
  const uintptr_t b = reinterpret_cast<uintptr_t>(base);
  const uintptr_t q = reinterpret_cast<uintptr_t>(ptr);
  const bool ok = q >= b && (q - b) % sizeof(T) == 0 && n >= 0 &&
                  int64_t((q - b) / sizeof(T)) <= count - n;
  return kat_check(ok);
#else
  (void)base; (void)count; (void)ptr; (void)n;
  return true;
#endif
}

__device__ __forceinline__ int64_t fast_div(int64_t n, uint64_t m, int32_t s1, int32_t s2) {
  const uint64_t un = uint64_t(n);
  const uint64_t t = __umul64hi(m, un);
  return int64_t((t + ((un - t) >> s1)) >> s2);
}

// Per-block, per-group reduction of one segment's per-thread sums (fixed order): thread t
// of the `nthreads` participants stores its 10 sums (slot-major, rows padded by one float so
// the slots fall in different banks), then each output (local group x slot) is added in
// fp64 over the tile's rows and its group's columns — by a warp with a fixed lane split and
// xor tree when a group spans more than 32 values, else by one thread in order — and written
// to the block's workspace slot.  kNamed selects a named barrier over the participants (warp-specialised
// kernels) instead of __syncthreads.
template <bool kNamed>
__device__ __forceinline__ void participants_sync(int nthreads) {
  if constexpr (kNamed) {
    asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
  } else {
    __syncthreads();
  }
}

template <bool kNamed>
__device__ __forceinline__ void segment_reduce(const float (&sums)[kAcc], float* s_acc,
                                               int stride, int tid, int nthreads, const Plan& p,
                                               int64_t cb, int64_t seg, int64_t blk,
                                               double* __restrict__ partial) {
#pragma unroll
  for (int k = 0; k < kAcc; ++k) s_acc[k * stride + tid] = sums[k];
  participants_sync<kNamed>(nthreads);
  const int64_t col0 = cb * p.tile_cols;
  const int64_t col_end = min(col0 + p.tile_cols, p.vec_cols);
  const int64_t g_first = col0 / p.vec_group;
  const int64_t g_last = (col_end - 1) / p.vec_group;
  const int n_out = int(g_last - g_first + 1) * kAcc;
  const int64_t span = min(int64_t(p.tile_cols), p.vec_group) * p.tile_rows;
  const int64_t ws_count = int64_t(p.workspace_bytes / sizeof(double));
  kat_check(seg >= 0 && seg < p.max_segments && g_last - g_first < p.max_local_groups &&
            stride >= p.tile_rows * p.tile_cols && nthreads <= stride);
  if (span > 32) {
    // Wide groups: warp w adds outputs w, w + nwarps, ...; lane j takes columns j, j+32, ...
    // of every row, then a fixed xor tree.
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int nwarps = nthreads >> 5;
    for (int o = warp; o < n_out; o += nwarps) {
      const int lg = o / kAcc;
      const int k = o - lg * kAcc;
      const int64_t g = g_first + lg;
      const int tlo = int(max(g * p.vec_group, col0) - col0);
      const int thi = int(min((g + 1) * p.vec_group, col_end) - col0);
      double v = 0.0;
      const float* base = s_acc + k * stride;
      for (int r = 0; r < p.tile_rows; ++r) {
        const float* row = base + r * p.tile_cols;
        for (int c = tlo + lane; c < thi; c += 32) v += double(row[c]);
      }
#pragma unroll
      for (int m = 16; m > 0; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
      double* dst = partial + ((blk * p.max_segments + seg) * p.max_local_groups + lg) * kAcc + k;
      if (lane == 0 && in_bounds(partial, ws_count, dst)) *dst = v;
    }
  } else {
    // Narrow groups: thread o adds output o = (local group, slot) over its rows and columns.
    for (int o = tid; o < n_out; o += nthreads) {
      const int lg = o / kAcc;
      const int k = o - lg * kAcc;
      const int64_t g = g_first + lg;
      const int tlo = int(max(g * p.vec_group, col0) - col0);
      const int thi = int(min((g + 1) * p.vec_group, col_end) - col0);
      double v = 0.0;
      const float* base = s_acc + k * stride;
      for (int r = 0; r < p.tile_rows; ++r) {
        const float* row = base + r * p.tile_cols;
        for (int c = tlo; c < thi; ++c) v += double(row[c]);
      }
      double* dst = partial + ((blk * p.max_segments + seg) * p.max_local_groups + lg) * kAcc + k;
      if (in_bounds(partial, ws_count, dst)) *dst = v;
    }
  }
  participants_sync<kNamed>(nthreads);
}

// ---------------------------------------------------------------------------
// Forward kernel.
// ---------------------------------------------------------------------------

// Rows handled by thread row `tr` inside a segment start at r0 and step by tile_rows;
// they are processed U at a time, and the next U rows are loaded before the current
// ones are computed, so every thread keeps loads in flight while it computes.
template <typename Tio, int V, int U, int kF>
__global__ void __launch_bounds__(kMaxThreads)
kat_fwd_kernel(const Tio* __restrict__ x, Tio* __restrict__ y,
               const float* __restrict__ num, const float* __restrict__ den, const Plan p) {
  using L = typename std::conditional<V == 1, float, float2>::type;
  using Raw = typename RawOf<Tio, V>::T;
  constexpr bool kExact = sizeof(Tio) == 4;
  const int tc = threadIdx.x % p.tile_cols;
  const int tr = threadIdx.x / p.tile_cols;
  if (tr >= p.tile_rows) return;
  // Programmatic dependent of the previous kernel on the stream: wait for it before reading.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  int64_t i0, i1;
  block_items(p, blockIdx.x, i0, i1);
  const int64_t step = int64_t(p.tile_rows) * p.width;
  for (int64_t i = i0; i < i1;) {
    const int64_t cb = i / p.rows;
    const int64_t seg_end = min(i1, (cb + 1) * p.rows);
    const int64_t col = cb * p.tile_cols + tc;
    const int64_t r0 = i - cb * p.rows + tr;
    const int64_t r_end = seg_end - cb * p.rows;
    if (col < p.vec_cols && r0 < r_end) {
      FwdCoef<L> c;
      load_fwd_coef<L, kF>(num, den, col / p.vec_group, c, p.num_stride);
      const int64_t n = (r_end - r0 + p.tile_rows - 1) / p.tile_rows;
      const Tio* xp = x + r0 * p.width + col * V;
      Tio* yp = y + r0 * p.width + col * V;
      const int64_t n_elems = p.rows * p.width;
      Raw cur[U];
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (u < n && in_bounds(x, n_elems, xp + u * step, V)) cur[u] = load_raw<Tio, V>(xp + u * step);
      xp += U * step;
#pragma unroll 1
      for (int64_t b = 0; b < n; b += U) {
        Raw nxt[U];
#pragma unroll
        for (int u = 0; u < U; ++u)
          if (b + U + u < n && in_bounds(x, n_elems, xp + u * step, V))
            nxt[u] = load_raw<Tio, V>(xp + u * step);
#pragma unroll
        for (int u = 0; u < U; ++u)
          if (b + u < n && in_bounds(y, n_elems, yp + u * step, V))
            store_raw<Tio, V>(yp + u * step, fwd_vec<Tio, V, L, kExact, kF>(cur[u], c));
#pragma unroll
        for (int u = 0; u < U; ++u) cur[u] = nxt[u];
        xp += U * step;
        yp += U * step;
      }
    }
    i = seg_end;
  }
}

// ---------------------------------------------------------------------------
// Backward kernel (dx + per-block partial coefficient sums).
// ---------------------------------------------------------------------------

template <typename Tio, int V, int U, int kF>
__global__ void __launch_bounds__(kMaxThreads)
kat_bwd_kernel(const Tio* __restrict__ x, const Tio* __restrict__ gy, Tio* __restrict__ dx,
               const float* __restrict__ num, const float* __restrict__ den,
               double* __restrict__ partial, const Plan p) {
  using L = typename std::conditional<V == 1, float, float2>::type;
  using Raw = typename RawOf<Tio, V>::T;
  constexpr bool kRefine = sizeof(Tio) == 4;
  __shared__ float s_acc[kAcc][kMaxThreads + 1];

  const int tc = threadIdx.x % p.tile_cols;
  const int tr = threadIdx.x / p.tile_cols;
  const bool row_thread = tr < p.tile_rows;
  const bool write_dx = dx != nullptr;

  int64_t i0, i1;
  block_items(p, blockIdx.x, i0, i1);
  const int64_t step = int64_t(p.tile_rows) * p.width;
  const int64_t cb0 = i0 / p.rows;

  for (int64_t i = i0; i < i1;) {
    const int64_t cb = i / p.rows;
    const int64_t seg_end = min(i1, (cb + 1) * p.rows);
    const int64_t col = cb * p.tile_cols + tc;
    L acc[kAcc];
#pragma unroll
    for (int k = 0; k < kAcc; ++k) acc[k] = bcast<L>(0.0f);

    const int64_t r0 = i - cb * p.rows + tr;
    const int64_t r_end = seg_end - cb * p.rows;
    if (row_thread && col < p.vec_cols && r0 < r_end) {
      BwdCoef<L> c;
      load_bwd_coef<L, kF>(num, den, col / p.vec_group, c, p.num_stride);
      const int64_t n = (r_end - r0 + p.tile_rows - 1) / p.tile_rows;
      const int64_t off = r0 * p.width + col * V;
      const Tio* xp = x + off;
      const Tio* gp = gy + off;
      Tio* dp = write_dx ? dx + off : nullptr;
      const int64_t n_elems = p.rows * p.width;
      Raw cx[U], cg[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (u < n && in_bounds(x, n_elems, xp + u * step, V) &&
            in_bounds(gy, n_elems, gp + u * step, V)) {
          cx[u] = load_raw<Tio, V>(xp + u * step);
          cg[u] = load_raw<Tio, V>(gp + u * step);
        }
      }
      xp += U * step;
      gp += U * step;
#pragma unroll 1
      for (int64_t b = 0; b < n; b += U) {
        Raw nx[U], ng[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          if (b + U + u < n && in_bounds(x, n_elems, xp + u * step, V) &&
              in_bounds(gy, n_elems, gp + u * step, V)) {
            nx[u] = load_raw<Tio, V>(xp + u * step);
            ng[u] = load_raw<Tio, V>(gp + u * step);
          }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          if (b + u < n) {
            const Raw d = bwd_vec<Tio, V, L, kRefine, kF>(cx[u], cg[u], c, acc);
            if (write_dx && in_bounds(dx, n_elems, dp + u * step, V))
              store_raw<Tio, V>(dp + u * step, d);
          }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          cx[u] = nx[u];
          cg[u] = ng[u];
        }
        xp += U * step;
        gp += U * step;
        if (write_dx) dp += U * step;
      }
    }

    // Block reduction of this segment, per group, in a fixed order.
    float sums[kAcc];
#pragma unroll
    for (int k = 0; k < kAcc; ++k) sums[k] = lane_sum(acc[k]);
    segment_reduce<false>(sums, &s_acc[0][0], kMaxThreads + 1, threadIdx.x, blockDim.x, p, cb,
                          cb - cb0, blockIdx.x, partial);
    i = seg_end;
  }
}

// ---------------------------------------------------------------------------
// Backward with a per-thread cp.async ring (16-byte vectors).
//
// Each thread streams its own future vectors of x and grad_out into a private ring of
// kStages slots (kRows rows each) in shared memory with cp.async (16-byte, L1-bypassing,
// 256-byte L2 fetch), one commit group per batch, and reads a batch back once
// cp.async.wait_group shows it landed.  Loads in flight live in shared memory instead of
// registers, so two blocks fit per SM and each keeps (kStages - 1) batches in flight.
// Slot layout: [stage][row][tensor][thread] of 16-byte vectors (conflict-free).
// ---------------------------------------------------------------------------

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global.L2::256B [%0], [%1], 16;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
               "l"(gmem_src)
               : "memory");
}
// 8-byte variant (the .cg form copies 16 bytes only): for groups whose width allows 8-byte
// vectors but not 16-byte ones.
__device__ __forceinline__ void cp_async8(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
               "l"(gmem_src)
               : "memory");
}
template <int kVB>
__device__ __forceinline__ void cp_async_vec(void* smem_dst, const void* gmem_src) {
  if constexpr (kVB == 16) cp_async16(smem_dst, gmem_src); else cp_async8(smem_dst, gmem_src);
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Block size cap of the cp.async backward (one block per SM at 512 threads x 128 registers).
#ifndef KAT_ASYNC_THREADS
#define KAT_ASYNC_THREADS 512
#endif
constexpr int kAsyncThreads = KAT_ASYNC_THREADS;
#ifndef KAT_ASYNC_MAXNREG
#define KAT_ASYNC_MAXNREG 0
#endif
#if KAT_ASYNC_MAXNREG > 0
#define KAT_ASYNC_BOUNDS __maxnreg__(KAT_ASYNC_MAXNREG)
#else
#define KAT_ASYNC_BOUNDS __launch_bounds__(kAsyncThreads)
#endif

template <typename Tio, int kStages, int kRows, int kF, int kVB = 16>
__global__ void KAT_ASYNC_BOUNDS
kat_bwd_async_kernel(const Tio* __restrict__ x, const Tio* __restrict__ gy, Tio* __restrict__ dx,
                     const float* __restrict__ num, const float* __restrict__ den,
                     double* __restrict__ partial, const Plan p) {
  constexpr int V = kVB / sizeof(Tio);   // elements per vector (16- or 8-byte vectors)
  constexpr bool kRefine = sizeof(Tio) == 4;
  using L = typename std::conditional<sizeof(Tio) == 4, S2, float2>::type;
  using Slot = typename BitsOf<kVB>::T;
  extern __shared__ __align__(16) uint4 ring_words[];
  Slot* const ring = reinterpret_cast<Slot*>(ring_words);
  const int T = blockDim.x;
  float* s_acc = reinterpret_cast<float*>(ring + size_t(kStages) * kRows * 2 * T);
  // Programmatic dependent of the previous kernel on the stream: wait for it before reading.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int tid = threadIdx.x;
  const int tc = tid % p.tile_cols;
  const int tr = tid / p.tile_cols;
  const bool row_thread = tr < p.tile_rows;
  const bool write_dx = dx != nullptr;
  int64_t i0, i1;
  block_items(p, blockIdx.x, i0, i1);
  const int64_t step = int64_t(p.tile_rows) * p.width;
  const int64_t cb0 = i0 / p.rows;
  Slot* const ring_t = ring + tid;
  const int slot_stride = 2 * T;            // slots between rows of a stage
  const int stage_stride = kRows * 2 * T;   // slots between stages

  for (int64_t i = i0; i < i1;) {
    const int64_t cb = i / p.rows;
    const int64_t seg_end = min(i1, (cb + 1) * p.rows);
    const int64_t col = cb * p.tile_cols + tc;
    const int64_t r0 = i - cb * p.rows + tr;
    const int64_t r_end = seg_end - cb * p.rows;
    L acc[kAcc];
#pragma unroll
    for (int k = 0; k < kAcc; ++k) acc[k] = bcast<L>(0.0f);
    if (row_thread && col < p.vec_cols && r0 < r_end) {
      BwdCoef<L> c;
      load_bwd_coef<L, kF>(num, den, col / p.vec_group, c, p.num_stride);
      const int n = int(min(int64_t(0x7fffffff), (r_end - r0 + p.tile_rows - 1) / p.tile_rows));
      const int nb = (n + kRows - 1) / kRows;
      const int64_t off = r0 * p.width + col * V;
      const Tio* lx = x + off;   // next rows to load
      const Tio* lg = gy + off;
      Tio* dp = write_dx ? dx + off : nullptr;
      const int64_t n_elems = p.rows * p.width;
      int load_stage = 0;
      int load_row = 0;
      // Issue the loads of the next batch (rows load_row .. load_row + kRows - 1).
      auto issue = [&]() {
        Slot* sp = ring_t + load_stage * stage_stride;
#pragma unroll
        for (int u = 0; u < kRows; ++u) {
          if (load_row + u < n) {
            if (in_bounds(x, n_elems, lx, V) && in_bounds(gy, n_elems, lg, V)) {
              cp_async_vec<kVB>(sp + u * slot_stride, lx);
              cp_async_vec<kVB>(sp + u * slot_stride + T, lg);
            }
            lx += step;
            lg += step;
          }
        }
        load_row += kRows;
        load_stage = load_stage + 1 == kStages ? 0 : load_stage + 1;
        cp_async_commit();
      };
#pragma unroll
      for (int b = 0; b < kStages - 1; ++b) issue();
      int use_stage = 0;
#pragma unroll 1
      for (int b = 0; b < nb; ++b) {
        issue();
        cp_async_wait<kStages - 1>();
        const Slot* sp = ring_t + use_stage * stage_stride;
#pragma unroll
        for (int u = 0; u < kRows; ++u) {
          if (b * kRows + u < n) {
            const Slot rx = sp[u * slot_stride];
            const Slot rg = sp[u * slot_stride + T];
            const Slot d = bwd_vec<Tio, V, L, kRefine, kF>(rx, rg, c, acc);
            if (write_dx) {
              if (in_bounds(dx, n_elems, dp, V)) store_raw<Tio, V>(dp, d);
              dp += step;
            }
          }
        }
        use_stage = use_stage + 1 == kStages ? 0 : use_stage + 1;
      }
      cp_async_wait<0>();
    }
    float sums[kAcc];
#pragma unroll
    for (int k = 0; k < kAcc; ++k) sums[k] = lane_sum(acc[k]);
    segment_reduce<false>(sums, s_acc, T + 1, tid, T, p, cb, cb - cb0, blockIdx.x, partial);
    i = seg_end;
  }
}

// Sum of group g's 10 coefficient slots over all blocks of the grid, computed by one warp:
// lane j takes blocks j, j+32, ... in order (each block's segments in order), then the 10
// lane totals are added with a fixed xor tree, leaving the result in every lane.  The segments
// of a block that hold group g are the column blocks cb0 .. cb1 of the block's item range that
// meet the group's vector columns; the loads of kAhead consecutive blocks of a lane are issued
// before any of them is added, so a lane waits for memory once per kAhead blocks, and a
// block's further segments of the group are loaded kSegAhead at a time.  The order of the
// additions is the block order, then the segment order, whatever the two depths: they only set
// how many loads are in flight (DepthOneSegment / DepthSegments below; launch_reduce picks one
// per plan).
__device__ __forceinline__ const double* group_slot(const double* __restrict__ partial,
                                                    const Plan& p, int64_t blk, int64_t seg,
                                                    int64_t lg) {
  const double* src = partial + ((blk * p.max_segments + seg) * p.max_local_groups + lg) * kAcc;
  if (!kat_check(seg < p.max_segments && lg < p.max_local_groups) ||
      !in_bounds(partial, int64_t(p.workspace_bytes / sizeof(double)), src, kAcc))
    return nullptr;
  return src;
}

template <int kAhead, int kSegAhead>
__device__ __forceinline__ void group_totals(const double* __restrict__ partial, const Plan& p,
                                             int64_t g, int lane, double (&tot)[kAcc]) {
#pragma unroll
  for (int k = 0; k < kAcc; ++k) tot[k] = 0.0;
  // column blocks that meet group g's vector columns [g vg, (g + 1) vg)
  const int64_t cb_lo = (g * p.vec_group) / p.tile_cols;
  const int64_t cb_hi = ((g + 1) * p.vec_group - 1) / p.tile_cols;
  for (int64_t b0 = lane; b0 < p.blocks; b0 += 32 * kAhead) {
    int64_t lo[kAhead], hi[kAhead], c0[kAhead];
    const double* first[kAhead];
    double v[kAhead][kAcc];
#pragma unroll
    for (int a = 0; a < kAhead; ++a) {
      const int64_t blk = b0 + 32 * a;
      first[a] = nullptr;
      lo[a] = 1;
      hi[a] = 0;
      c0[a] = 0;
      if (blk < p.blocks) {
        int64_t i0, i1;
        block_items(p, blk, i0, i1);
        c0[a] = fast_div(i0, p.rows_m, p.rows_s1, p.rows_s2);
        const int64_t c1 = fast_div(i1 - 1, p.rows_m, p.rows_s1, p.rows_s2);
        lo[a] = max(c0[a], cb_lo);
        hi[a] = min(c1, cb_hi);
        if (lo[a] <= hi[a]) {
          const int64_t gf = fast_div(lo[a] * p.tile_cols, p.vg_m, p.vg_s1, p.vg_s2);
          first[a] = group_slot(partial, p, blk, lo[a] - c0[a], g - gf);
        }
      }
#pragma unroll
      for (int k = 0; k < kAcc; ++k) v[a][k] = first[a] != nullptr ? first[a][k] : 0.0;
    }
#pragma unroll
    for (int a = 0; a < kAhead; ++a) {
      if (first[a] == nullptr) continue;
#pragma unroll
      for (int k = 0; k < kAcc; ++k) tot[k] += v[a][k];
      // further column blocks of this block that hold part of the group (wide groups): their
      // loads are issued kSegAhead at a time before any of them is added, still added in
      // column-block order
      for (int64_t cb = lo[a] + 1; cb <= hi[a]; cb += kSegAhead) {
        double w[kSegAhead][kAcc];
        bool have[kSegAhead];
#pragma unroll
        for (int s = 0; s < kSegAhead; ++s) {
          const double* src = nullptr;
          if (cb + s <= hi[a]) {
            const int64_t gf = fast_div((cb + s) * p.tile_cols, p.vg_m, p.vg_s1, p.vg_s2);
            src = group_slot(partial, p, b0 + 32 * a, cb + s - c0[a], g - gf);
          }
          have[s] = src != nullptr;
#pragma unroll
          for (int k = 0; k < kAcc; ++k) w[s][k] = have[s] ? src[k] : 0.0;
        }
#pragma unroll
        for (int s = 0; s < kSegAhead; ++s) {
          if (!have[s]) continue;
#pragma unroll
          for (int k = 0; k < kAcc; ++k) tot[k] += w[s][k];
        }
      }
    }
  }
#pragma unroll
  for (int k = 0; k < kAcc; ++k) {
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) tot[k] += __shfl_xor_sync(0xffffffffu, tot[k], m);
  }
}

// Writes one group's gradients from its totals: d_num = sums; d_den = -sgn(b) * sums for
// the KAT formula (sgn(0) = 0 and sgn(NaN) = NaN, as torch.sgn), -sums for the abs-after-sum
// formula (whose per-element sign was applied in the sums).  Lane k < 10 writes slot k.
__device__ __forceinline__ void write_group(const double (&tot)[kAcc], double scale, bool ok,
                                            int64_t g, int lane, const float* __restrict__ den,
                                            float* __restrict__ dnum, float* __restrict__ dden,
                                            int formula) {
  double v = 0.0;
#pragma unroll
  for (int k = 0; k < kAcc; ++k)
    if (lane == k) v = tot[k];
  if (lane >= kAcc) return;
  const float f = ok ? float(v * scale) : __int_as_float(0x7fc00000);
  if (lane < 6) {
    dnum[g * 6 + lane] = f;
  } else {
    float sg = 1.0f;
    if (formula == kFormulaKat) {
      const float b = den[g * 4 + (lane - 6)];
      sg = b > 0.0f ? 1.0f : (b < 0.0f ? -1.0f : b * 0.0f);
    }
    dden[g * 4 + (lane - 6)] = -(sg * f);
  }
}

// Load depths of the grid reductions: with one segment per block (every block inside one
// column block, the usual case) five blocks per lane cover a 148-block grid in one round of
// loads; with several segments per block, four blocks and four further segments per round
// (x[64,256,56,56] NCHW: ~11 segments of a group per block).  Same additions, same bits.
struct DepthOneSegment { static constexpr int kAhead = 5, kSeg = 1; };
struct DepthSegments { static constexpr int kAhead = 4, kSeg = 4; };

// Grid reduction: one warp per group.
constexpr int kReduceWarps = 8;
template <typename Depth>
__global__ void __launch_bounds__(kReduceWarps * 32)
kat_bwd_reduce_kernel(const double* __restrict__ partial, const float* __restrict__ den,
                      float* __restrict__ dnum, float* __restrict__ dden, const Plan p) {
  const int64_t g = int64_t(blockIdx.x) * kReduceWarps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (g >= p.num_groups) return;
  // Launched as a programmatic dependent of the partial-sum kernel: wait here until that grid
  // has completed and its stores are visible (returns at once for an ordinary launch).
  asm volatile("griddepcontrol.wait;" ::: "memory");
  double tot[kAcc];
  group_totals<Depth::kAhead, Depth::kSeg>(partial, p, g, lane, tot);
  write_group(tot, 1.0, true, g, lane, den, dnum, dden, p.formula);
}

// The same with one numerator row shared by every group: one block; warp w takes groups
// w, w + 8, ... in order, writes their denominator gradients and adds their numerator totals;
// the 8 warp sums are then added in warp order (fp64) and rounded once into dnum[0..5].
template <typename Depth>
__global__ void __launch_bounds__(kReduceWarps * 32)
kat_bwd_reduce_shared_kernel(const double* __restrict__ partial, const float* __restrict__ den,
                             float* __restrict__ dnum, float* __restrict__ dden, const Plan p) {
  __shared__ double s_num[kReduceWarps][6];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  double num_sum = 0.0;   // lane k < 6: numerator moment k over this warp's groups
  for (int64_t g = warp; g < p.num_groups; g += kReduceWarps) {
    double tot[kAcc];
    group_totals<Depth::kAhead, Depth::kSeg>(partial, p, g, lane, tot);
#pragma unroll
    for (int k = 0; k < 6; ++k)
      if (lane == k) num_sum += tot[k];
    if (lane >= 6 && lane < kAcc) {
      double v = 0.0;
#pragma unroll
      for (int k = 6; k < kAcc; ++k)
        if (lane == k) v = tot[k];
      float sg = 1.0f;
      if (p.formula == kFormulaKat) {
        const float b = den[g * 4 + (lane - 6)];
        sg = b > 0.0f ? 1.0f : (b < 0.0f ? -1.0f : b * 0.0f);
      }
      dden[g * 4 + (lane - 6)] = -(sg * float(v));
    }
  }
  if (lane < 6) s_num[warp][lane] = num_sum;
  __syncthreads();
  if (threadIdx.x < 6) {
    double v = 0.0;
    for (int w = 0; w < kReduceWarps; ++w) v += s_num[w][threadIdx.x];
    dnum[threadIdx.x] = float(v);
  }
}

// ---------------------------------------------------------------------------
// Bulk-copy pipelined kernels (16-byte vectors).
//
// Warp 0 is the producer: one lane streams the block's tiles (stage_rows rows of its
// column block, for x and — backward — grad_out) from global memory into a ring of
// `stages` shared-memory slots with cp.async.bulk, each slot guarded by a "full"
// mbarrier (transaction-counted) and an "empty" mbarrier (one arrival per consumer
// warp).  The other warps consume: each thread keeps its fixed vector column, reads its
// vectors from shared memory, computes, and stores y / dx straight to global memory.
// The ring keeps up to stages x stage bytes of loads in flight per SM without holding
// them in registers.  Every wait is bounded (about two seconds of clock cycles); a wait
// that runs out sets the block's abort flag and the sticky device status word, and the
// block then runs to completion without further waiting.
// ---------------------------------------------------------------------------

struct Pipe {
  int32_t stages;       // ring depth
  int32_t stage_rows;   // rows per slot (multiple of tile_rows)
  int32_t seg_bytes;    // bytes of one row slot = tile_cols * 16
  int32_t contiguous;   // 1: a slot is one contiguous global range per tensor
  uint32_t smem_bytes;  // dynamic shared memory per block
  uint32_t chunk_bytes; // largest single bulk copy (multiple of 16)
  int32_t poll_ns;      // < 0: every lane polls; >= 0: lane 0 polls with this back-off
};

constexpr int kStatusWaitTimeout = 1;
constexpr long long kWaitCycles = 4000000000LL;
constexpr uint32_t kPipeHeader = 256;  // barriers + abort flag, keeps slots 128-byte aligned

__device__ __forceinline__ uint32_t smem_addr(const void* ptr) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(ptr));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}
// Slot release by a consumer warp.  Relaxed: the slot only guards this warp's shared-memory
// reads (complete once their values were used); a release arrive would also wait for the
// warp's preceding global stores to be performed.
__device__ __forceinline__ void mbar_arrive_relaxed(uint64_t* bar) {
  asm volatile("mbarrier.arrive.relaxed.cta.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar))
               : "memory");
}
// Non-suspending test of the phase with `parity` (mbarrier.test_wait): the waits below
// poll it, so a released slot is seen at once (try_wait may park the thread for a
// system-dependent time first).
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}
// Bulk global -> shared copy of `bytes` (multiple of 16, both addresses 16-byte aligned)
// completing as transactions on `bar`.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// Consumer-warp wait: lane 0 polls with a short back-off, then every lane observes the
// completed phase itself (acquire), so the bulk-copied data is visible to all lanes.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort);
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          int backoff_ns) {
  bool ok = true;
  if ((threadIdx.x & 31) == 0) {
    const long long t0 = clock64();
    while (!mbar_test(bar, parity)) {
      if (*abort) { ok = false; break; }
      if (clock64() - t0 > kWaitCycles) {
        *abort = 1;
        atomicExch(&g_kat_status, kStatusWaitTimeout);
        ok = false;
        break;
      }
      if (backoff_ns > 0) __nanosleep(backoff_ns);
    }
  }
  ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
  if (ok) mbar_wait(bar, parity, abort);
  return ok;
}

// Bounded wait for the phase with `parity` of `bar`.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  if (mbar_test(bar, parity)) return true;
  const long long t0 = clock64();
  for (;;) {
    if (mbar_test(bar, parity)) return true;
    if (*abort) return false;
    if (clock64() - t0 > kWaitCycles) {
      *abort = 1;
      atomicExch(&g_kat_status, kStatusWaitTimeout);
      return false;
    }
  }
}

// The block's tiles, in order: consecutive runs of up to stage_rows rows that stay in
// one column block.
struct TileCursor {
  int64_t i, i1;
  __device__ TileCursor(const Plan& p, int64_t blk) { block_items(p, blk, i, i1); }
  __device__ bool next(const Plan& p, int stage_rows, int64_t& cb, int64_t& row, int& nrows,
                       bool& seg_last) {
    if (i >= i1) return false;
    cb = i / p.rows;
    row = i - cb * p.rows;
    const int64_t seg_end = min(i1, (cb + 1) * p.rows);
    const int64_t n = min(int64_t(stage_rows), seg_end - i);
    nrows = int(n);
    i += n;
    seg_last = i == seg_end;
    return true;
  }
};

// Producer lane: stream the block's tiles of `kTensors` inputs into the ring.
template <typename Tio, int kTensors>
__device__ __forceinline__ void produce(const Tio* __restrict__ in0, const Tio* __restrict__ in1,
                                        const Plan& p, const Pipe& q, uint64_t* full,
                                        uint64_t* empty, char* slots, volatile int* abort) {
  constexpr int V = 16 / sizeof(Tio);
  TileCursor cur(p, blockIdx.x);
  int64_t cb, row;
  int nrows;
  bool last;
  const uint32_t slot_bytes = uint32_t(q.stage_rows) * uint32_t(q.seg_bytes);
  for (uint32_t k = 0; cur.next(p, q.stage_rows, cb, row, nrows, last); ++k) {
    const uint32_t s = k % uint32_t(q.stages);
    if (k >= uint32_t(q.stages) && !mbar_wait(&empty[s], ((k / q.stages) - 1) & 1u, abort)) break;
    const int64_t col0 = cb * p.tile_cols;
    const uint32_t row_bytes = uint32_t(min(int64_t(p.tile_cols), p.vec_cols - col0)) * 16u;
    {
      // The tile's first and last element of every tensor, and its slot, in range.
      const int64_t n_elems = p.rows * p.width;
      const int64_t first = row * p.width + col0 * V;
      const int64_t last_end = (row + nrows - 1) * p.width + col0 * V + row_bytes / sizeof(Tio);
      const bool ok = in_bounds(in0, n_elems, in0 + first, last_end - first) &&
                      (kTensors == 1 || in_bounds(in1, n_elems, in1 + first, last_end - first)) &&
                      kat_check(uint32_t(nrows) <= uint32_t(q.stage_rows) &&
                                row_bytes <= uint32_t(q.seg_bytes));
      if (!ok) {
        *abort = 1;
        break;
      }
    }
    mbar_arrive_expect_tx(&full[s], row_bytes * uint32_t(nrows) * kTensors);
#pragma unroll
    for (int t = 0; t < kTensors; ++t) {
      const Tio* base = (t == 0 ? in0 : in1) + row * p.width + col0 * V;
      char* dst = slots + (size_t(s) * kTensors + t) * slot_bytes;
      if (q.contiguous) {
        const char* src = reinterpret_cast<const char*>(base);
        const uint32_t total = row_bytes * uint32_t(nrows);
        for (uint32_t off = 0; off < total; off += q.chunk_bytes)
          bulk_load(dst + off, src + off, min(q.chunk_bytes, total - off), &full[s]);
      } else {
        for (int j = 0; j < nrows; ++j) {
          const char* src = reinterpret_cast<const char*>(base + int64_t(j) * p.width);
          char* d = dst + size_t(j) * q.seg_bytes;
          for (uint32_t off = 0; off < row_bytes; off += q.chunk_bytes)
            bulk_load(d + off, src + off, min(q.chunk_bytes, row_bytes - off), &full[s]);
        }
      }
    }
  }
}

__device__ __forceinline__ void pipe_init(uint64_t* full, uint64_t* empty, volatile int* abort,
                                          int stages, int consumer_warps) {
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], uint32_t(consumer_warps));
    }
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
}

template <typename Tio>
__global__ void __launch_bounds__(kMaxThreads + 32)
kat_fwd_tma_kernel(const Tio* __restrict__ x, Tio* __restrict__ y, const float* __restrict__ num,
                   const float* __restrict__ den, const Plan p, const Pipe q) {
  constexpr int V = 16 / sizeof(Tio);
  using Raw = uint4;
  constexpr bool kExact = sizeof(Tio) == 4;
  extern __shared__ __align__(128) char smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + q.stages;
  volatile int* abort = reinterpret_cast<volatile int*>(empty + q.stages);
  char* slots = smem + kPipeHeader;
  const int consumer_warps = int(blockDim.x >> 5) - 1;
  pipe_init(full, empty, abort, q.stages, consumer_warps);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (warp == 0) {
    if (lane == 0) produce<Tio, 1>(x, nullptr, p, q, full, empty, slots, abort);
    return;
  }
  const int ctid = threadIdx.x - 32;
  const int tc = ctid % p.tile_cols;
  const int tr = ctid / p.tile_cols;
  const bool row_thread = tr < p.tile_rows;
  const uint32_t slot_bytes = uint32_t(q.stage_rows) * uint32_t(q.seg_bytes);
  TileCursor cur(p, blockIdx.x);
  int64_t cb, row, cb_coef = -1;
  int nrows;
  bool last;
  FwdCoef<float2> c;
  for (uint32_t k = 0; cur.next(p, q.stage_rows, cb, row, nrows, last); ++k) {
    const uint32_t s = k % uint32_t(q.stages);
    if (q.poll_ns < 0) mbar_wait(&full[s], (k / q.stages) & 1u, abort);
    else warp_wait(&full[s], (k / q.stages) & 1u, abort, q.poll_ns);
    const int64_t col = cb * p.tile_cols + tc;
    if (row_thread && col < p.vec_cols) {
      if (cb != cb_coef) {
        load_fwd_coef<float2, kFormulaKat>(num, den, col / p.vec_group, c, p.num_stride);
        cb_coef = cb;
      }
      const char* src = slots + size_t(s) * slot_bytes + size_t(tc) * 16;
      Tio* dst = y + row * p.width + col * V;
      for (int j = tr; j < nrows; j += p.tile_rows) {
        const Raw raw = *reinterpret_cast<const Raw*>(src + size_t(j) * q.seg_bytes);
        if (in_bounds(y, p.rows * p.width, dst + int64_t(j) * p.width, V))
          store_raw<Tio, V>(dst + int64_t(j) * p.width, fwd_vec<Tio, V, float2, kExact>(raw, c));
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive_relaxed(&empty[s]);
  }
}

template <typename Tio>
__global__ void __launch_bounds__(kMaxThreads + 32)
kat_bwd_tma_kernel(const Tio* __restrict__ x, const Tio* __restrict__ gy, Tio* __restrict__ dx,
                   const float* __restrict__ num, const float* __restrict__ den,
                   double* __restrict__ partial, const Plan p, const Pipe q) {
  constexpr int V = 16 / sizeof(Tio);
  using Raw = uint4;
  constexpr bool kRefine = sizeof(Tio) == 4;
  extern __shared__ __align__(128) char smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + q.stages;
  volatile int* abort = reinterpret_cast<volatile int*>(empty + q.stages);
  char* slots = smem + kPipeHeader;
  const uint32_t slot_bytes = uint32_t(q.stage_rows) * uint32_t(q.seg_bytes);
  float* s_acc = reinterpret_cast<float*>(slots + size_t(q.stages) * 2 * slot_bytes);
  const int consumer_warps = int(blockDim.x >> 5) - 1;
  pipe_init(full, empty, abort, q.stages, consumer_warps);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (warp == 0) {
    if (lane == 0) produce<Tio, 2>(x, gy, p, q, full, empty, slots, abort);
    return;
  }
  const int nthreads = consumer_warps * 32;
  const int ctid = threadIdx.x - 32;
  const int tc = ctid % p.tile_cols;
  const int tr = ctid / p.tile_cols;
  const bool row_thread = tr < p.tile_rows;
  const bool write_dx = dx != nullptr;
  int64_t i0, i1;
  block_items(p, blockIdx.x, i0, i1);
  const int64_t cb0 = i0 / p.rows;
  TileCursor cur(p, blockIdx.x);
  int64_t cb, row, cb_coef = -1;
  int nrows;
  bool last;
  BwdCoef<float2> c;
  float2 acc[kAcc];
#pragma unroll
  for (int k = 0; k < kAcc; ++k) acc[k] = make_float2(0.0f, 0.0f);
  for (uint32_t k = 0; cur.next(p, q.stage_rows, cb, row, nrows, last); ++k) {
    const uint32_t s = k % uint32_t(q.stages);
    if (q.poll_ns < 0) mbar_wait(&full[s], (k / q.stages) & 1u, abort);
    else warp_wait(&full[s], (k / q.stages) & 1u, abort, q.poll_ns);
    const int64_t col = cb * p.tile_cols + tc;
    if (row_thread && col < p.vec_cols) {
      if (cb != cb_coef) {
        load_bwd_coef<float2, kFormulaKat>(num, den, col / p.vec_group, c, p.num_stride);
        cb_coef = cb;
      }
      const char* xs = slots + (size_t(s) * 2) * slot_bytes + size_t(tc) * 16;
      const char* gs = xs + slot_bytes;
      Tio* dst = write_dx ? dx + row * p.width + col * V : nullptr;
      for (int j = tr; j < nrows; j += p.tile_rows) {
        const Raw rx = *reinterpret_cast<const Raw*>(xs + size_t(j) * q.seg_bytes);
        const Raw rg = *reinterpret_cast<const Raw*>(gs + size_t(j) * q.seg_bytes);
        const Raw d = bwd_vec<Tio, V, float2, kRefine>(rx, rg, c, acc);
        if (write_dx && in_bounds(dx, p.rows * p.width, dst + int64_t(j) * p.width, V))
          store_raw<Tio, V>(dst + int64_t(j) * p.width, d);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive_relaxed(&empty[s]);
    if (last) {
      float sums[kAcc];
#pragma unroll
      for (int a = 0; a < kAcc; ++a) {
        sums[a] = lane_sum(acc[a]);
        acc[a] = make_float2(0.0f, 0.0f);
      }
      segment_reduce<true>(sums, s_acc, nthreads + 1, ctid, nthreads, p, cb, cb - cb0,
                           blockIdx.x, partial);
    }
  }
}

// ---------------------------------------------------------------------------
// Grid reduction fused with the cross-GPU exchange (data parallel over NVLink).
//
// One block: (1) sums every (group, slot) over the blocks of this GPU exactly as
// kat_bwd_reduce_kernel does; (2) stores the G x 10 fp64 sums into every rank's exchange
// buffer (peer memory, NVLink stores), into the row of this rank in the half selected by
// the call's epoch parity; (3) waits, bounded by a wall-clock limit, until every rank's row on
// this GPU carries this call's tag; (4) adds the ranks in rank order in fp64 (optionally
// divided by the world size) and writes d_num / d_den.  All ranks add the same numbers in
// the same order, so their gradients are bit-identical.
//
// Tagged words.  Each fp64 sum travels as two 8-byte words, each holding 32 bits of the value
// and the 32-bit tag of the call (the low half of its epoch).  An aligned 8-byte store is
// single-copy atomic, so a reader sees a word either before the store or whole after it: a
// word with the right tag carries the right data.  No fence and no separate flag are needed,
// and every thread of the block waits for its own words in parallel (relaxed system-scope
// stores and loads).
//
// The epoch is a per-buffer counter the kernel increments, so calls must be made the same
// number of times on every rank (each rank's k-th call pairs with every other rank's k-th
// call).  Two epoch halves let a rank run ahead by one call without overwriting data a peer
// still reads: a rank can post call e + 1 only after it saw every row of call e, and call
// e + 2 only after every rank posted e + 1, which a rank does only once it has read its call-e
// inbox.  So a word of the half being read carries the tag of call e or of call e - 2 (not yet
// overwritten); any other tag means the pairing broke.
//
// Failure is fail-stop.  A wait that runs out, or a word with a tag out of step, sets
// KAT_DEVICE_EXCHANGE_TIMEOUT in the device status word, writes NaN gradients and sets this
// rank's `broken` word; every later call on a broken buffer writes NaN at once and stores
// nothing to any peer.  A rank that gave up therefore never posts again, so a late peer can
// only pair with data that was really posted for its call (it gets correct sums once, then
// times out itself) and no rank ever adds data of two different calls.  Only local memory is
// written after a failure: a peer that has gone away is never touched again.  The buffer
// stays broken until it is rebuilt.
//
// Exchange buffer layout (every rank, zero-initialised once):
//   [0]    u64 epoch     [8] u64 broken
//   [128]  u64 inbox[2][kMaxPeers][G * 10 * 2]   word = tag << 32 | 32 bits of a sum
// ---------------------------------------------------------------------------

constexpr int kMaxPeers = 8;
constexpr size_t kExchangeHeader = 128;
constexpr int kStatusExchangeTimeout = 2;

struct Peers {
  int32_t world;
  int32_t rank;
  int32_t average;
  int32_t timeout_ms;
  char* buf[kMaxPeers];
};

__device__ __forceinline__ void st_relaxed_sys(uint64_t* ptr, uint64_t v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(ptr), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_sys(const uint64_t* ptr) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(ptr) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// The exchange itself, called by every thread of one block: s_sum[0 .. n_out) holds this
// rank's sums on entry and the rank-order fp64 sums over all ranks on return (true), or the
// call failed (false: timeout, tag out of step or a broken buffer; the status word is set).
__device__ bool exchange_rows(double* s_sum, int n_out, const Peers& peers) {
  __shared__ uint64_t s_epoch;
  __shared__ int s_ok;
  __shared__ volatile int s_fail;
  const int tid = threadIdx.x;
  const int n_words = 2 * n_out;      // tagged words per rank row
  char* const own = peers.buf[peers.rank];
  uint64_t* const broken = reinterpret_cast<uint64_t*>(own + 8);
  if (tid == 0) {
    uint64_t* ep = reinterpret_cast<uint64_t*>(own);
    s_ok = *broken == 0 ? 1 : 0;
    s_fail = 0;
    s_epoch = *ep + 1;
    if (s_ok) *ep = s_epoch;
    else atomicExch(&g_kat_status, kStatusExchangeTimeout);
  }
  __syncthreads();
  const uint64_t epoch = s_epoch;
  const uint32_t tag = uint32_t(epoch);
  const uint32_t stale = uint32_t(epoch - 2);   // the tag this half held before (0 = never written)
  const int64_t half_words = int64_t(kMaxPeers) * n_words;
  const int64_t inbox_words = 2 * half_words;
  const size_t half = size_t(epoch & 1u);
  const uint64_t* mine = reinterpret_cast<const uint64_t*>(own + kExchangeHeader) +
                         half * half_words;
  if (s_ok) {
    // this rank's row into every rank's inbox: value bits low / high with the tag
    for (int r = 0; r < peers.world; ++r) {
      uint64_t* inbox = reinterpret_cast<uint64_t*>(peers.buf[r] + kExchangeHeader);
      uint64_t* dst = inbox + half * half_words + int64_t(peers.rank) * n_words;
      if (!in_bounds(inbox, inbox_words, dst, n_words)) continue;
      for (int i = tid; i < n_words; i += blockDim.x) {
        const uint64_t bits = uint64_t(__double_as_longlong(s_sum[i >> 1]));
        const uint32_t word = (i & 1) ? uint32_t(bits >> 32) : uint32_t(bits);
        st_relaxed_sys(dst + i, (uint64_t(tag) << 32) | word);
      }
    }
    // every word of every rank's row of this half carries this call's tag
    const uint64_t limit = uint64_t(peers.timeout_ms) * 1000000ull;
    const uint64_t t0 = global_timer_ns();
    const int total = peers.world * n_words;
    for (int j = tid; j < total && !s_fail; j += blockDim.x) {
      const uint64_t* w = mine + j;   // rank j / n_words, word j % n_words (rows adjacent)
      for (;;) {
        const uint32_t t = uint32_t(ld_relaxed_sys(w) >> 32);
        if (t == tag) break;
        const bool in_step = t == stale || (epoch <= 2 && t == 0);
        if (!in_step || s_fail || global_timer_ns() - t0 > limit) {
          s_fail = 1;
          break;
        }
        __nanosleep(32);
      }
    }
  }
  __syncthreads();   // every thread is done with its own row and with the waits
  const bool ok = s_ok && !s_fail;
  if (tid == 0 && s_ok && s_fail) {
    *broken = 1;
    atomicExch(&g_kat_status, kStatusExchangeTimeout);
  }
  if (ok) {
    // ranks added in rank order, in fp64
    for (int i = tid; i < n_out; i += blockDim.x) {
      double v = 0.0;
      for (int q = 0; q < peers.world; ++q) {
        const uint64_t* row = mine + int64_t(q) * n_words;
        const uint64_t lo = ld_relaxed_sys(row + 2 * i) & 0xffffffffull;
        const uint64_t hi = ld_relaxed_sys(row + 2 * i + 1) & 0xffffffffull;
        v += __longlong_as_double((long long)(lo | (hi << 32)));
      }
      s_sum[i] = v;
    }
  }
  __syncthreads();
  return ok;
}

__global__ void __launch_bounds__(kReduceThreads, 1)
kat_bwd_reduce_exchange_kernel(const double* __restrict__ partial, const float* __restrict__ den,
                               float* __restrict__ dnum, float* __restrict__ dden, const Plan p,
                               const Peers peers) {
  extern __shared__ double s_sum[];   // [G * 10]
  const int G = int(p.num_groups);
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int nwarps = blockDim.x >> 5;
  // Programmatic dependent of the partial-sum kernel, as kat_bwd_reduce_kernel.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  for (int g = warp; g < G; g += nwarps) {
    double tot[kAcc];
    group_totals<4, 1>(partial, p, g, lane, tot);
#pragma unroll
    for (int k = 0; k < kAcc; ++k)
      if (lane == k) s_sum[g * kAcc + k] = tot[k];
  }
  __syncthreads();
  const bool ok = exchange_rows(s_sum, G * kAcc, peers);
  const double scale = peers.average ? 1.0 / double(peers.world) : 1.0;
  const bool shared = p.num_stride == 0;   // one numerator row: its gradient summed over groups
  for (int g = warp; g < G; g += nwarps) {
    double tot[kAcc];
#pragma unroll
    for (int k = 0; k < kAcc; ++k) tot[k] = s_sum[g * kAcc + k];
    if (!shared || lane >= 6) write_group(tot, scale, ok, g, lane, den, dnum, dden, p.formula);
  }
  if (shared && tid < 6) {
    // the order of kat_bwd_reduce_shared_kernel: groups w, w + 8, ... per warp w, then warps
    double v = 0.0;
    for (int w = 0; w < kReduceWarps; ++w) {
      double a = 0.0;
      for (int g = w; g < G; g += kReduceWarps) a += s_sum[g * kAcc + tid];
      v += a;
    }
    dnum[tid] = ok ? float(v * scale) : __int_as_float(0x7fc00000);
  }
}

// Exchange-only call: this rank's final coefficient gradients (fp32, [G, 6] and [G, 4]) in,
// the rank-order fp64 sum over all ranks (optionally averaged), rounded once, out (in place).
__global__ void __launch_bounds__(kReduceThreads, 1)
kat_exchange_grads_kernel(float* __restrict__ dnum, float* __restrict__ dden, int G,
                          const Peers peers) {
  extern __shared__ double s_sum[];   // [G * 10]: d_num row g then d_den row g
  const int n_out = G * kAcc;
  for (int i = threadIdx.x; i < n_out; i += blockDim.x) {
    const int g = i / kAcc, k = i - g * kAcc;
    s_sum[i] = double(k < 6 ? dnum[g * 6 + k] : dden[g * 4 + (k - 6)]);
  }
  __syncthreads();
  const bool ok = exchange_rows(s_sum, n_out, peers);
  const double scale = peers.average ? 1.0 / double(peers.world) : 1.0;
  for (int i = threadIdx.x; i < n_out; i += blockDim.x) {
    const int g = i / kAcc, k = i - g * kAcc;
    const float f = ok ? float(s_sum[i] * scale) : __int_as_float(0x7fc00000);
    if (k < 6) dnum[g * 6 + k] = f;
    else dden[g * 4 + (k - 6)] = f;
  }
}

// ---------------------------------------------------------------------------
// Host side: validation, planning, dispatch.
// ---------------------------------------------------------------------------

#ifndef KAT_FWD_UNROLL
#define KAT_FWD_UNROLL 4
#endif
#ifndef KAT_BWD_UNROLL
#define KAT_BWD_UNROLL 2
#endif
constexpr int kUnroll = KAT_FWD_UNROLL;
constexpr int kUnrollBwd = KAT_BWD_UNROLL;


// Programmatic dependent launch: the forward, the cp.async backward and the grid reductions are
// launched with programmatic stream serialization, so each can be launched while the previous
// kernel on the stream drains; each waits (griddepcontrol.wait) before it reads anything.
// KAT_RATIONAL_PDL=0 launches them as ordinary stream-ordered kernels.
bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("KAT_RATIONAL_PDL");
    return !(e != nullptr && e[0] == '0');
  }();
  return on;
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

void to_public(const Plan& p, kat_rational_plan* out) {
  out->rows = p.rows;
  out->width = p.width;
  out->group_width = p.group_width;
  out->num_groups = p.num_groups;
  out->vec = p.vec;
  out->threads = p.threads;
  out->tile_cols = p.tile_cols;
  out->tile_rows = p.tile_rows;
  out->col_blocks = p.col_blocks;
  out->items = p.items;
  out->blocks = p.blocks;
  out->max_segments = p.max_segments;
  out->max_local_groups = p.max_local_groups;
  out->workspace_bytes = p.workspace_bytes;
  out->col_block_blocks = p.cb_q;
  out->col_block_extra = p.cb_r;
}

// Per-device SM count and per-(device, kernel, block size) occupancy caches.
std::mutex g_cache_mu;
std::map<int, int> g_sm_count;
std::map<std::tuple<int, const void*, int>, int> g_occupancy;

cudaError_t device_sm_count(int dev, int* out) {
  std::lock_guard<std::mutex> lock(g_cache_mu);
  auto it = g_sm_count.find(dev);
  if (it != g_sm_count.end()) {
    *out = it->second;
    return cudaSuccess;
  }
  int v = 0;
  cudaError_t e = cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  g_sm_count[dev] = v;
  *out = v;
  return cudaSuccess;
}

cudaError_t kernel_occupancy(int dev, const void* fn, int threads, int* out) {
  std::lock_guard<std::mutex> lock(g_cache_mu);
  auto key = std::make_tuple(dev, fn, threads);
  auto it = g_occupancy.find(key);
  if (it != g_occupancy.end()) {
    *out = it->second;
    return cudaSuccess;
  }
  int v = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, fn, threads, 0);
  if (e != cudaSuccess) return e;
  if (v < 1) v = 1;
  g_occupancy[key] = v;
  *out = v;
  return cudaSuccess;
}

// Kernel selection by (dtype, vec, formula).
template <int kF>
const void* fwd_kernel_for_f(int dtype, int vec) {
  switch (dtype) {
    case KAT_DTYPE_F32:
      switch (vec) {
        case 4: return (const void*)kat_fwd_kernel<float, 4, kUnroll, kF>;
        case 2: return (const void*)kat_fwd_kernel<float, 2, kUnroll, kF>;
        default: return (const void*)kat_fwd_kernel<float, 1, kUnroll, kF>;
      }
    case KAT_DTYPE_F16:
      switch (vec) {
        case 8: return (const void*)kat_fwd_kernel<__half, 8, kUnroll, kF>;
        case 4: return (const void*)kat_fwd_kernel<__half, 4, kUnroll, kF>;
        case 2: return (const void*)kat_fwd_kernel<__half, 2, kUnroll, kF>;
        default: return (const void*)kat_fwd_kernel<__half, 1, kUnroll, kF>;
      }
    default:
      switch (vec) {
        case 8: return (const void*)kat_fwd_kernel<__nv_bfloat16, 8, kUnroll, kF>;
        case 4: return (const void*)kat_fwd_kernel<__nv_bfloat16, 4, kUnroll, kF>;
        case 2: return (const void*)kat_fwd_kernel<__nv_bfloat16, 2, kUnroll, kF>;
        default: return (const void*)kat_fwd_kernel<__nv_bfloat16, 1, kUnroll, kF>;
      }
  }
}

template <int kF>
const void* bwd_kernel_for_f(int dtype, int vec) {
  switch (dtype) {
    case KAT_DTYPE_F32:
      switch (vec) {
        case 4: return (const void*)kat_bwd_kernel<float, 4, kUnrollBwd, kF>;
        case 2: return (const void*)kat_bwd_kernel<float, 2, kUnrollBwd, kF>;
        default: return (const void*)kat_bwd_kernel<float, 1, kUnrollBwd, kF>;
      }
    case KAT_DTYPE_F16:
      switch (vec) {
        case 8: return (const void*)kat_bwd_kernel<__half, 8, kUnrollBwd, kF>;
        case 4: return (const void*)kat_bwd_kernel<__half, 4, kUnrollBwd, kF>;
        case 2: return (const void*)kat_bwd_kernel<__half, 2, kUnrollBwd, kF>;
        default: return (const void*)kat_bwd_kernel<__half, 1, kUnrollBwd, kF>;
      }
    default:
      switch (vec) {
        case 8: return (const void*)kat_bwd_kernel<__nv_bfloat16, 8, kUnrollBwd, kF>;
        case 4: return (const void*)kat_bwd_kernel<__nv_bfloat16, 4, kUnrollBwd, kF>;
        case 2: return (const void*)kat_bwd_kernel<__nv_bfloat16, 2, kUnrollBwd, kF>;
        default: return (const void*)kat_bwd_kernel<__nv_bfloat16, 1, kUnrollBwd, kF>;
      }
  }
}

const void* fwd_kernel_for(int dtype, int vec, int formula) {
  return formula == kFormulaKat ? fwd_kernel_for_f<kFormulaKat>(dtype, vec)
                                : fwd_kernel_for_f<kFormulaAbsSum>(dtype, vec);
}

const void* bwd_kernel_for(int dtype, int vec, int formula) {
  return formula == kFormulaKat ? bwd_kernel_for_f<kFormulaKat>(dtype, vec)
                                : bwd_kernel_for_f<kFormulaAbsSum>(dtype, vec);
}

// Widest vector the shape and every (non-NULL) pointer allow.
int pick_vec(int dtype, int64_t group_width, const void* const* ptrs, int n_ptrs) {
  int vec = max_vec_for(dtype);
  const int eb = elem_bytes(dtype);
  for (;;) {
    if (vec == 1) return 1;
    bool ok = group_width % vec == 0;
    for (int i = 0; ok && i < n_ptrs; ++i)
      if (ptrs[i] != nullptr && (reinterpret_cast<uintptr_t>(ptrs[i]) % uintptr_t(vec * eb)) != 0)
        ok = false;
    if (ok) return vec;
    vec >>= 1;
  }
}

// Plans are pure functions of (device, kernel family, shape, dtype, vector width) once the
// device's SM count and the kernel's occupancy are known; cache them so repeated calls on
// the same shape skip the planning arithmetic and the cache lookups it makes.
struct PlanKey {
  int dev;
  const void* fn;   // the kernel the plan is for
  int dtype, vec;
  int64_t batch, channels, inner, groups;
  bool operator<(const PlanKey& o) const {
    return std::tie(dev, fn, dtype, vec, batch, channels, inner, groups) <
           std::tie(o.dev, o.fn, o.dtype, o.vec, o.batch, o.channels, o.inner, o.groups);
  }
};
struct PlanEntry {
  int status;
  Plan plan;
  Pipe pipe;
};
std::mutex g_plan_mu;
std::map<PlanKey, PlanEntry> g_plan_cache;
constexpr size_t kPlanCacheMax = 4096;

bool plan_cache_get(const PlanKey& k, PlanEntry* e) {
  std::lock_guard<std::mutex> lock(g_plan_mu);
  auto it = g_plan_cache.find(k);
  if (it == g_plan_cache.end()) return false;
  *e = it->second;
  return true;
}
void plan_cache_put(const PlanKey& k, const PlanEntry& e) {
  std::lock_guard<std::mutex> lock(g_plan_mu);
  if (g_plan_cache.size() >= kPlanCacheMax) g_plan_cache.clear();
  g_plan_cache[k] = e;
}

int plan_for_launch_uncached(const void* fn, int64_t batch, int64_t channels, int64_t inner,
                             int64_t num_groups, int dtype, int vec, Plan* p);

int plan_for_launch(const void* fn, int64_t batch, int64_t channels, int64_t inner,
                    int64_t num_groups, int dtype, int vec, Plan* p) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return KAT_ERR_CUDA;
  const PlanKey key{dev, fn, dtype, vec, batch, channels, inner, num_groups};
  PlanEntry e;
  if (plan_cache_get(key, &e)) {
    *p = e.plan;
    return e.status;
  }
  e.status = plan_for_launch_uncached(fn, batch, channels, inner, num_groups, dtype, vec, &e.plan);
  if (e.status == KAT_OK) plan_cache_put(key, e);
  *p = e.plan;
  return e.status;
}

int plan_for_launch_uncached(const void* fn, int64_t batch, int64_t channels, int64_t inner,
                             int64_t num_groups, int dtype, int vec, Plan* p) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return KAT_ERR_CUDA;
  int sms = 0;
  if (device_sm_count(dev, &sms) != cudaSuccess) return KAT_ERR_CUDA;
  // The block size depends only on the shape; plan once with occupancy 1 to get it.
  Plan probe;
  int st = make_plan_impl(batch, channels, inner, num_groups, dtype, vec, sms, 1, &probe);
  if (st != KAT_OK) return st;
  int occ = 1;
  if (kernel_occupancy(dev, fn, probe.threads, &occ) != cudaSuccess) return KAT_ERR_CUDA;
  return make_plan_impl(batch, channels, inner, num_groups, dtype, vec, sms, occ, p);
}

template <typename Tio, int V, int kF>
cudaError_t launch_fwd_t(const void* x, void* y, const float* num, const float* den, const Plan& p,
                         cudaStream_t s) {
  return launch_pdl(kat_fwd_kernel<Tio, V, kUnroll, kF>, dim3(unsigned(p.blocks)),
                    dim3(unsigned(p.threads)), 0, s, static_cast<const Tio*>(x),
                    static_cast<Tio*>(y), num, den, p);
}

template <typename Tio, int V, int kF>
cudaError_t launch_bwd_t(const void* x, const void* gy, void* dx, const float* num,
                         const float* den, double* partial, const Plan& p, cudaStream_t s) {
  kat_bwd_kernel<Tio, V, kUnrollBwd, kF><<<dim3(unsigned(p.blocks)), dim3(unsigned(p.threads)), 0, s>>>(
      static_cast<const Tio*>(x), static_cast<const Tio*>(gy), static_cast<Tio*>(dx), num, den,
      partial, p);
  return cudaGetLastError();
}

template <int kF>
cudaError_t launch_fwd_f(int dtype, int vec, const void* x, void* y, const float* num,
                       const float* den, const Plan& p, cudaStream_t s) {
  switch (dtype) {
    case KAT_DTYPE_F32:
      if (vec == 4) return launch_fwd_t<float, 4, kF>(x, y, num, den, p, s);
      if (vec == 2) return launch_fwd_t<float, 2, kF>(x, y, num, den, p, s);
      return launch_fwd_t<float, 1, kF>(x, y, num, den, p, s);
    case KAT_DTYPE_F16:
      if (vec == 8) return launch_fwd_t<__half, 8, kF>(x, y, num, den, p, s);
      if (vec == 4) return launch_fwd_t<__half, 4, kF>(x, y, num, den, p, s);
      if (vec == 2) return launch_fwd_t<__half, 2, kF>(x, y, num, den, p, s);
      return launch_fwd_t<__half, 1, kF>(x, y, num, den, p, s);
    default:
      if (vec == 8) return launch_fwd_t<__nv_bfloat16, 8, kF>(x, y, num, den, p, s);
      if (vec == 4) return launch_fwd_t<__nv_bfloat16, 4, kF>(x, y, num, den, p, s);
      if (vec == 2) return launch_fwd_t<__nv_bfloat16, 2, kF>(x, y, num, den, p, s);
      return launch_fwd_t<__nv_bfloat16, 1, kF>(x, y, num, den, p, s);
  }
}

template <int kF>
cudaError_t launch_bwd_f(int dtype, int vec, const void* x, const void* gy, void* dx,
                       const float* num, const float* den, double* partial, const Plan& p,
                       cudaStream_t s) {
  switch (dtype) {
    case KAT_DTYPE_F32:
      if (vec == 4) return launch_bwd_t<float, 4, kF>(x, gy, dx, num, den, partial, p, s);
      if (vec == 2) return launch_bwd_t<float, 2, kF>(x, gy, dx, num, den, partial, p, s);
      return launch_bwd_t<float, 1, kF>(x, gy, dx, num, den, partial, p, s);
    case KAT_DTYPE_F16:
      if (vec == 8) return launch_bwd_t<__half, 8, kF>(x, gy, dx, num, den, partial, p, s);
      if (vec == 4) return launch_bwd_t<__half, 4, kF>(x, gy, dx, num, den, partial, p, s);
      if (vec == 2) return launch_bwd_t<__half, 2, kF>(x, gy, dx, num, den, partial, p, s);
      return launch_bwd_t<__half, 1, kF>(x, gy, dx, num, den, partial, p, s);
    default:
      if (vec == 8) return launch_bwd_t<__nv_bfloat16, 8, kF>(x, gy, dx, num, den, partial, p, s);
      if (vec == 4) return launch_bwd_t<__nv_bfloat16, 4, kF>(x, gy, dx, num, den, partial, p, s);
      if (vec == 2) return launch_bwd_t<__nv_bfloat16, 2, kF>(x, gy, dx, num, den, partial, p, s);
      return launch_bwd_t<__nv_bfloat16, 1, kF>(x, gy, dx, num, den, partial, p, s);
  }
}

cudaError_t launch_fwd(int dtype, int vec, int formula, const void* x, void* y,
                       const float* num, const float* den, const Plan& p, cudaStream_t s) {
  return formula == kFormulaKat ? launch_fwd_f<kFormulaKat>(dtype, vec, x, y, num, den, p, s)
                                : launch_fwd_f<kFormulaAbsSum>(dtype, vec, x, y, num, den, p, s);
}

cudaError_t launch_bwd(int dtype, int vec, int formula, const void* x, const void* gy, void* dx,
                       const float* num, const float* den, double* partial, const Plan& p,
                       cudaStream_t s) {
  return formula == kFormulaKat
             ? launch_bwd_f<kFormulaKat>(dtype, vec, x, gy, dx, num, den, partial, p, s)
             : launch_bwd_f<kFormulaAbsSum>(dtype, vec, x, gy, dx, num, den, partial, p, s);
}

// ----- Bulk-copy pipeline: planning and launch --------------------------------

constexpr int kPipeSmemBudget = 200 * 1024;

// Tuning knobs (environment, read once): slot size per input tensor, ring depth cap and
// largest single bulk copy.
int env_int(const char* name, int dflt) {
  const char* e = getenv(name);
  if (e == nullptr || *e == 0) return dflt;
  const long v = strtol(e, nullptr, 10);
  return v > 0 ? int(v) : dflt;
}
int stage_target_bytes() {
  static const int v = env_int("KAT_RATIONAL_STAGE_BYTES", 16 * 1024);
  return v;
}
int max_stages() {
  static const int v = std::min(env_int("KAT_RATIONAL_STAGES", 8), 8);
  return v;
}
int poll_mode_ns() {
  static const int v = [] {
    const char* e = getenv("KAT_RATIONAL_POLL_NS");
    return (e == nullptr || *e == 0) ? -1 : int(strtol(e, nullptr, 10));
  }();
  return v;
}
int tma_ctas_per_sm() {
  static const int v = std::min(env_int("KAT_RATIONAL_TMA_CTAS", 1), 4);
  return v;
}
uint32_t bulk_chunk_bytes() {
  static const uint32_t v = uint32_t(env_int("KAT_RATIONAL_BULK_CHUNK", 1 << 20)) & ~15u;
  return v < 16 ? 16 : v;
}

// KAT_RATIONAL_PIPELINE selects how 16-byte-vector problems stream their inputs (a
// tuning switch; every choice computes the same results):
//   unset / "async"  forward: register prefetch; backward: per-thread cp.async ring
//   "registers"      register prefetch for both
//   "bulk"           producer-warp cp.async.bulk ring for both
int pipeline_mode() {
  static const int mode = [] {
    const char* e = getenv("KAT_RATIONAL_PIPELINE");
    if (e != nullptr && strcmp(e, "registers") == 0) return 1;
    if (e != nullptr && strcmp(e, "bulk") == 0) return 2;
    return 0;
  }();
  return mode;
}
bool bulk_pipeline_enabled() { return pipeline_mode() == 2; }

// Slot geometry for a plan made with 16-byte vectors.  Returns false when no ring of at
// least two slots fits in shared memory.
bool make_pipe(const Plan& p, int tensors, bool bwd, Pipe* q) {
  if (p.items == 0) return false;
  q->seg_bytes = p.tile_cols * 16;
  const int64_t group_bytes = int64_t(q->seg_bytes) * p.tile_rows;
  int64_t rows = stage_target_bytes() / group_bytes;
  if (rows < 1) rows = 1;
  q->stage_rows = int32_t(rows * p.tile_rows);
  const int64_t acc_bytes = bwd ? int64_t(kAcc) * (p.threads + 1) * 4 : 0;
  const int64_t budget = kPipeSmemBudget / tma_ctas_per_sm() - kPipeHeader - acc_bytes;
  int64_t stage_bytes = int64_t(q->stage_rows) * q->seg_bytes * tensors;
  int64_t stages = budget / stage_bytes;
  if (stages < 2) {
    q->stage_rows = p.tile_rows;
    stage_bytes = int64_t(q->stage_rows) * q->seg_bytes * tensors;
    stages = budget / stage_bytes;
    if (stages < 2) return false;
  }
  if (stages > max_stages()) stages = max_stages();
  if (stage_bytes >= (1 << 20)) return false;  // mbarrier transaction-count range
  q->stages = int32_t(stages);
  q->contiguous = (p.col_blocks == 1 && int64_t(p.tile_cols) == p.vec_cols) ? 1 : 0;
  q->smem_bytes = uint32_t(kPipeHeader + stages * stage_bytes + acc_bytes);
  q->chunk_bytes = bulk_chunk_bytes();
  q->poll_ns = poll_mode_ns();
  return true;
}

std::map<std::pair<int, const void*>, bool> g_smem_attr;

cudaError_t allow_dynamic_smem(int dev, const void* fn, uint32_t bytes) {
  std::lock_guard<std::mutex> lock(g_cache_mu);
  auto key = std::make_pair(dev, fn);
  if (g_smem_attr.count(key)) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       kPipeSmemBudget);
  if (e != cudaSuccess) return e;
  (void)bytes;
  g_smem_attr[key] = true;
  return cudaSuccess;
}

const void* fwd_tma_kernel_for(int dtype) {
  switch (dtype) {
    case KAT_DTYPE_F32: return (const void*)kat_fwd_tma_kernel<float>;
    case KAT_DTYPE_F16: return (const void*)kat_fwd_tma_kernel<__half>;
    default: return (const void*)kat_fwd_tma_kernel<__nv_bfloat16>;
  }
}

const void* bwd_tma_kernel_for(int dtype) {
  switch (dtype) {
    case KAT_DTYPE_F32: return (const void*)kat_bwd_tma_kernel<float>;
    case KAT_DTYPE_F16: return (const void*)kat_bwd_tma_kernel<__half>;
    default: return (const void*)kat_bwd_tma_kernel<__nv_bfloat16>;
  }
}

// Plan + slot geometry of the pipelined kernels (one block per SM).  Returns KAT_OK,
// an error, or -1 when the pipelined kernels do not apply to this shape.
int plan_tma_uncached(int64_t batch, int64_t channels, int64_t inner, int64_t num_groups,
                      int dtype, bool bwd, int* dev_out, Plan* p, Pipe* q);

int plan_tma(int64_t batch, int64_t channels, int64_t inner, int64_t num_groups, int dtype,
             bool bwd, int* dev_out, Plan* p, Pipe* q) {
  if (!bulk_pipeline_enabled()) return -1;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return KAT_ERR_CUDA;
  const PlanKey key{dev, bwd ? bwd_tma_kernel_for(dtype) : fwd_tma_kernel_for(dtype), dtype,
                    max_vec_for(dtype), batch, channels, inner, num_groups};
  PlanEntry e;
  if (!plan_cache_get(key, &e)) {
    e.status = plan_tma_uncached(batch, channels, inner, num_groups, dtype, bwd, dev_out, &e.plan,
                                 &e.pipe);
    if (e.status == KAT_OK || e.status == -1) plan_cache_put(key, e);
  }
  *dev_out = dev;
  *p = e.plan;
  *q = e.pipe;
  return e.status;
}

int plan_tma_uncached(int64_t batch, int64_t channels, int64_t inner, int64_t num_groups,
                      int dtype, bool bwd, int* dev_out, Plan* p, Pipe* q) {
  const int vmax = max_vec_for(dtype);
  const int64_t gw = (channels / num_groups) * inner;
  if (!bulk_pipeline_enabled() || gw % vmax != 0) return -1;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return KAT_ERR_CUDA;
  int sms = 0;
  if (device_sm_count(dev, &sms) != cudaSuccess) return KAT_ERR_CUDA;
  const int st = make_plan_impl(batch, channels, inner, num_groups, dtype, vmax, sms,
                                tma_ctas_per_sm(), p);
  if (st != KAT_OK) return st;
  if (!make_pipe(*p, bwd ? 2 : 1, bwd, q)) return -1;
  *dev_out = dev;
  return KAT_OK;
}

template <typename Tio>
cudaError_t launch_fwd_tma_t(const void* x, void* y, const float* num, const float* den,
                             const Plan& p, const Pipe& q, cudaStream_t s) {
  kat_fwd_tma_kernel<Tio><<<dim3(unsigned(p.blocks)), dim3(unsigned(p.threads + 32)),
                            q.smem_bytes, s>>>(static_cast<const Tio*>(x), static_cast<Tio*>(y),
                                               num, den, p, q);
  return cudaGetLastError();
}

template <typename Tio>
cudaError_t launch_bwd_tma_t(const void* x, const void* gy, void* dx, const float* num,
                             const float* den, double* partial, const Plan& p, const Pipe& q,
                             cudaStream_t s) {
  kat_bwd_tma_kernel<Tio><<<dim3(unsigned(p.blocks)), dim3(unsigned(p.threads + 32)),
                            q.smem_bytes, s>>>(
      static_cast<const Tio*>(x), static_cast<const Tio*>(gy), static_cast<Tio*>(dx), num, den,
      partial, p, q);
  return cudaGetLastError();
}

#ifndef KAT_ASYNC_STAGES
#define KAT_ASYNC_STAGES 4
#endif
#ifndef KAT_ASYNC_ROWS
#define KAT_ASYNC_ROWS 2
#endif
#ifndef KAT_ASYNC_COLS
#define KAT_ASYNC_COLS 128
#endif
constexpr int kAsyncCols = KAT_ASYNC_COLS;
constexpr int kAsyncStages = KAT_ASYNC_STAGES;
constexpr int kAsyncRows = KAT_ASYNC_ROWS;

size_t async_smem_bytes(int threads, int vec_bytes) {
  return size_t(kAsyncStages) * kAsyncRows * 2 * vec_bytes * threads +
         size_t(kAcc) * 4 * (threads + 1);
}

template <int kF, int kVB>
const void* bwd_async_kernel_for_fv(int dtype) {
  switch (dtype) {
    case KAT_DTYPE_F32:
      return (const void*)kat_bwd_async_kernel<float, kAsyncStages, kAsyncRows, kF, kVB>;
    case KAT_DTYPE_F16:
      return (const void*)kat_bwd_async_kernel<__half, kAsyncStages, kAsyncRows, kF, kVB>;
    default:
      return (const void*)kat_bwd_async_kernel<__nv_bfloat16, kAsyncStages, kAsyncRows, kF, kVB>;
  }
}

// The cp.async backward for (dtype, formula, vector bytes 16 or 8).
const void* bwd_async_kernel_for(int dtype, int formula, int vec_bytes = 16) {
  if (vec_bytes == 16)
    return formula == kFormulaKat ? bwd_async_kernel_for_fv<kFormulaKat, 16>(dtype)
                                  : bwd_async_kernel_for_fv<kFormulaAbsSum, 16>(dtype);
  return formula == kFormulaKat ? bwd_async_kernel_for_fv<kFormulaKat, 8>(dtype)
                                : bwd_async_kernel_for_fv<kFormulaAbsSum, 8>(dtype);
}

// Plan of the cp.async backward: occupancy from the kernel's registers and its shared
// memory at this block size.  Returns -1 when it does not apply.
int plan_async_uncached(int64_t batch, int64_t channels, int64_t inner, int64_t num_groups,
                        int dtype, int formula, int vec, int* dev_out, Plan* p);

// `vec` = elements per vector: max_vec_for(dtype) (16-byte vectors) or the 8-byte width.
int plan_async(int64_t batch, int64_t channels, int64_t inner, int64_t num_groups, int dtype,
               int formula, int* dev_out, Plan* p, int vec = 0) {
  if (pipeline_mode() != 0) return -1;
  if (vec == 0) vec = max_vec_for(dtype);
  const int vb = vec * elem_bytes(dtype);
  if (vb != 16 && vb != 8) return -1;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return KAT_ERR_CUDA;
  const PlanKey key{dev, bwd_async_kernel_for(dtype, formula, vb), dtype, vec, batch, channels,
                    inner, num_groups};
  PlanEntry e;
  if (!plan_cache_get(key, &e)) {
    e.status = plan_async_uncached(batch, channels, inner, num_groups, dtype, formula, vec,
                                   dev_out, &e.plan);
    if (e.status == KAT_OK || e.status == -1) plan_cache_put(key, e);
  }
  *dev_out = dev;
  *p = e.plan;
  return e.status;
}

int plan_async_uncached(int64_t batch, int64_t channels, int64_t inner, int64_t num_groups,
                        int dtype, int formula, int vec, int* dev_out, Plan* p) {
  const int vmax = vec;
  const int vb = vec * elem_bytes(dtype);
  const int64_t gw = (channels / num_groups) * inner;
  if (pipeline_mode() != 0 || gw % vmax != 0) return -1;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return KAT_ERR_CUDA;
  int sms = 0;
  if (device_sm_count(dev, &sms) != cudaSuccess) return KAT_ERR_CUDA;
  // Block shape of the cp.async backward: at most max_cols vector columns, and as many rows as
  // fill kAsyncThreads threads (at 128 registers, one 512-thread block per SM).  kAsyncCols
  // (128 columns x 4 rows) unless a wider tile of full blocks needs fewer ring refills
  // (refill_overhead, by more than 2% of a thread's rows): short, wide problems such as
  // x[64,256,56,56] NCHW, whose blocks cross ~11 column blocks of 64 rows at 128 columns
  // (backward 140 us there against 111 us at 512 columns on one B200).  KAT_RATIONAL_ASYNC_COLS
  // pins the width.
  static const int env_cols = env_int("KAT_RATIONAL_ASYNC_COLS", 0);
  int max_cols = kAsyncCols;
  Plan probe;
  int st = KAT_OK;
  if (env_cols > 0) {
    max_cols = std::max(32, std::min(env_cols, kAsyncThreads) / 32 * 32);
    st = make_plan_impl(batch, channels, inner, num_groups, dtype, vmax, sms, 1, &probe,
                        max_cols, kAsyncThreads);
  } else {
    st = make_plan_impl(batch, channels, inner, num_groups, dtype, vmax, sms, 1, &probe,
                        max_cols, kAsyncThreads);
    if (st != KAT_OK) return st;
    double best = refill_overhead(probe);
    for (int cols = 2 * kAsyncCols; cols <= kAsyncThreads; cols *= 2) {
      Plan wide;
      if (make_plan_impl(batch, channels, inner, num_groups, dtype, vmax, sms, 1, &wide, cols,
                         kAsyncThreads) != KAT_OK ||
          wide.threads != probe.threads)
        continue;
      const double ov = refill_overhead(wide);
      if (ov < best - 0.02) {
        best = ov;
        max_cols = cols;
        probe = wide;
      }
    }
  }
  if (st != KAT_OK) return st;
  const void* fn = bwd_async_kernel_for(dtype, formula, vb);
  const size_t smem = async_smem_bytes(probe.threads, vb);
  if (smem > size_t(kPipeSmemBudget)) return -1;
  if (allow_dynamic_smem(dev, fn, uint32_t(smem)) != cudaSuccess) return KAT_ERR_CUDA;
  int occ = 1;
  {
    std::lock_guard<std::mutex> lock(g_cache_mu);
    auto key = std::make_tuple(dev, fn, probe.threads);
    auto it = g_occupancy.find(key);
    if (it != g_occupancy.end()) {
      occ = it->second;
    } else {
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, probe.threads, smem) !=
          cudaSuccess)
        return KAT_ERR_CUDA;
      if (occ < 1) occ = 1;
      g_occupancy[key] = occ;
    }
  }
  st = make_plan_impl(batch, channels, inner, num_groups, dtype, vmax, sms, occ, p, max_cols,
                      kAsyncThreads);
  *dev_out = dev;
  return st;
}

template <typename Tio, int kF>
cudaError_t launch_bwd_async_t(const void* x, const void* gy, void* dx, const float* num,
                               const float* den, double* partial, const Plan& p, cudaStream_t s) {
  const int vb = p.vec * int(sizeof(Tio));
  if (vb == 16)
    return launch_pdl(kat_bwd_async_kernel<Tio, kAsyncStages, kAsyncRows, kF, 16>,
                      dim3(unsigned(p.blocks)), dim3(unsigned(p.threads)),
                      async_smem_bytes(p.threads, 16), s, static_cast<const Tio*>(x),
                      static_cast<const Tio*>(gy), static_cast<Tio*>(dx), num, den, partial, p);
  return launch_pdl(kat_bwd_async_kernel<Tio, kAsyncStages, kAsyncRows, kF, 8>,
                    dim3(unsigned(p.blocks)), dim3(unsigned(p.threads)),
                    async_smem_bytes(p.threads, 8), s, static_cast<const Tio*>(x),
                    static_cast<const Tio*>(gy), static_cast<Tio*>(dx), num, den, partial, p);
}

template <int kF>
cudaError_t launch_bwd_async_f(int dtype, const void* x, const void* gy, void* dx,
                               const float* num, const float* den, double* partial, const Plan& p,
                               cudaStream_t s) {
  switch (dtype) {
    case KAT_DTYPE_F32: return launch_bwd_async_t<float, kF>(x, gy, dx, num, den, partial, p, s);
    case KAT_DTYPE_F16: return launch_bwd_async_t<__half, kF>(x, gy, dx, num, den, partial, p, s);
    default: return launch_bwd_async_t<__nv_bfloat16, kF>(x, gy, dx, num, den, partial, p, s);
  }
}

cudaError_t launch_bwd_async(int dtype, int formula, const void* x, const void* gy, void* dx,
                             const float* num, const float* den, double* partial, const Plan& p,
                             cudaStream_t s) {
  return formula == kFormulaKat
             ? launch_bwd_async_f<kFormulaKat>(dtype, x, gy, dx, num, den, partial, p, s)
             : launch_bwd_async_f<kFormulaAbsSum>(dtype, x, gy, dx, num, den, partial, p, s);
}

cudaError_t launch_fwd_tma(int dtype, const void* x, void* y, const float* num, const float* den,
                           const Plan& p, const Pipe& q, cudaStream_t s) {
  switch (dtype) {
    case KAT_DTYPE_F32: return launch_fwd_tma_t<float>(x, y, num, den, p, q, s);
    case KAT_DTYPE_F16: return launch_fwd_tma_t<__half>(x, y, num, den, p, q, s);
    default: return launch_fwd_tma_t<__nv_bfloat16>(x, y, num, den, p, q, s);
  }
}

cudaError_t launch_bwd_tma(int dtype, const void* x, const void* gy, void* dx, const float* num,
                           const float* den, double* partial, const Plan& p, const Pipe& q,
                           cudaStream_t s) {
  switch (dtype) {
    case KAT_DTYPE_F32: return launch_bwd_tma_t<float>(x, gy, dx, num, den, partial, p, q, s);
    case KAT_DTYPE_F16: return launch_bwd_tma_t<__half>(x, gy, dx, num, den, partial, p, q, s);
    default: return launch_bwd_tma_t<__nv_bfloat16>(x, gy, dx, num, den, partial, p, q, s);
  }
}

int launch_reduce(const void* workspace, const float* den, float* dnum, float* dden,
                  const Plan& p, const Peers* peers, cudaStream_t s) {
  const bool one_segment = p.max_segments == 1;
  const double* partial = static_cast<const double*>(workspace);
  if (peers == nullptr && p.num_stride == 0) {
    const cudaError_t e =
        one_segment
            ? launch_pdl(kat_bwd_reduce_shared_kernel<DepthOneSegment>, dim3(1),
                         dim3(kReduceWarps * 32), 0, s, partial, den, dnum, dden, p)
            : launch_pdl(kat_bwd_reduce_shared_kernel<DepthSegments>, dim3(1),
                         dim3(kReduceWarps * 32), 0, s, partial, den, dnum, dden, p);
    if (e != cudaSuccess) return KAT_ERR_CUDA;
  } else if (peers == nullptr) {
    // Programmatic dependent launch: the reduction's launch overlaps the tail of the
    // partial-sum kernel, and griddepcontrol.wait inside it orders the reads.
    const unsigned grid = unsigned((p.num_groups + kReduceWarps - 1) / kReduceWarps);
    const cudaError_t e =
        one_segment ? launch_pdl(kat_bwd_reduce_kernel<DepthOneSegment>, dim3(grid),
                                 dim3(kReduceWarps * 32), 0, s, partial, den, dnum, dden, p)
                    : launch_pdl(kat_bwd_reduce_kernel<DepthSegments>, dim3(grid),
                                 dim3(kReduceWarps * 32), 0, s, partial, den, dnum, dden, p);
    if (e != cudaSuccess) return KAT_ERR_CUDA;
  } else {
    const size_t smem = size_t(p.num_groups) * kAcc * sizeof(double);
    if (smem > 48 * 1024) {
      if (cudaFuncSetAttribute((const void*)kat_bwd_reduce_exchange_kernel,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) !=
          cudaSuccess)
        return KAT_ERR_CUDA;
    }
    if (launch_pdl(kat_bwd_reduce_exchange_kernel, dim3(1), dim3(kReduceThreads), smem, s,
                   static_cast<const double*>(workspace), den, dnum, dden, p,
                   *peers) != cudaSuccess)
      return KAT_ERR_CUDA;
  }
  return cudaGetLastError() == cudaSuccess ? KAT_OK : KAT_ERR_CUDA;
}

// The backward: the fused elementwise/partial-sum kernel chosen for the shape, then the grid
// reduction — plain, or fused with the cross-GPU exchange when `peers` is given.
int bwd_impl(const void* x, const void* grad_out, void* grad_x, const float* numerator,
             const float* denominator, float* grad_numerator, float* grad_denominator,
             void* workspace, size_t workspace_bytes, int64_t batch, int64_t channels,
             int64_t inner, int64_t num_groups, int dtype, int formula, void* stream,
             const Peers* peers) {
  int64_t n = 0;
  int st = validate_dims(batch, channels, inner, num_groups, dtype, &n);
  if (st != KAT_OK) return st;
  const bool shared = (formula & KAT_SHARED_NUMERATOR) != 0;
  formula &= ~KAT_SHARED_NUMERATOR;
  if (formula != kFormulaKat && formula != kFormulaAbsSum) return KAT_ERR_BAD_FORMULA;
  if (peers != nullptr && formula != kFormulaKat) return KAT_ERR_BAD_FORMULA;
  const int num_stride = shared ? 0 : 6;
  if (numerator == nullptr || denominator == nullptr || grad_numerator == nullptr ||
      grad_denominator == nullptr)
    return KAT_ERR_NULL_POINTER;
  if (n != 0 && (x == nullptr || grad_out == nullptr)) return KAT_ERR_NULL_POINTER;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t gw = (channels / num_groups) * inner;
  const void* ptrs[3] = {x, grad_out, grad_x};
  const int vec = n == 0 ? 1 : pick_vec(dtype, gw, ptrs, 3);
  if (num_groups > 0x7fffffff) return KAT_ERR_BAD_GROUPS;
  Plan p;
  // cp.async backward for 16-byte and for 8-byte vectors.
  if (n != 0 && (vec == max_vec_for(dtype) || vec * elem_bytes(dtype) == 8)) {
    int dev = 0;
    st = plan_async(batch, channels, inner, num_groups, dtype, formula, &dev, &p, vec);
    if (st != -1) {
      if (st != KAT_OK) return st;
      if (workspace == nullptr || workspace_bytes < p.workspace_bytes ||
          (reinterpret_cast<uintptr_t>(workspace) % 16) != 0)
        return KAT_ERR_WORKSPACE;
      p.num_stride = num_stride;
      if (launch_bwd_async(dtype, formula, x, grad_out, grad_x, numerator, denominator,
                           static_cast<double*>(workspace), p, s) != cudaSuccess)
        return KAT_ERR_CUDA;
      p.formula = formula;
      return launch_reduce(workspace, denominator, grad_numerator, grad_denominator, p, peers, s);
    }
  }
  // The bulk-copy design computes the KAT formula only.
  if (n != 0 && vec == max_vec_for(dtype) && formula == kFormulaKat) {
    Pipe q;
    int dev = 0;
    st = plan_tma(batch, channels, inner, num_groups, dtype, true, &dev, &p, &q);
    if (st != -1) {
      if (st != KAT_OK) return st;
      if (workspace == nullptr || workspace_bytes < p.workspace_bytes ||
          (reinterpret_cast<uintptr_t>(workspace) % 16) != 0)
        return KAT_ERR_WORKSPACE;
      if (allow_dynamic_smem(dev, bwd_tma_kernel_for(dtype), q.smem_bytes) != cudaSuccess)
        return KAT_ERR_CUDA;
      p.num_stride = num_stride;
      if (launch_bwd_tma(dtype, x, grad_out, grad_x, numerator, denominator,
                         static_cast<double*>(workspace), p, q, s) != cudaSuccess)
        return KAT_ERR_CUDA;
      return launch_reduce(workspace, denominator, grad_numerator, grad_denominator, p, peers, s);
    }
  }
  if (n == 0) {
    st = make_plan_impl(batch, channels, inner, num_groups, dtype, vec, 1, 1, &p);
  } else {
    st = plan_for_launch(bwd_kernel_for(dtype, vec, formula), batch, channels, inner, num_groups,
                         dtype, vec, &p);
  }
  if (st != KAT_OK) return st;
  p.num_stride = num_stride;
  if (p.blocks > 0) {
    if (workspace == nullptr || workspace_bytes < p.workspace_bytes ||
        (reinterpret_cast<uintptr_t>(workspace) % 16) != 0)
      return KAT_ERR_WORKSPACE;
    if (launch_bwd(dtype, vec, formula, x, grad_out, grad_x, numerator, denominator,
                   static_cast<double*>(workspace), p, s) != cudaSuccess)
      return KAT_ERR_CUDA;
  }
  p.formula = formula;
  return launch_reduce(workspace, denominator, grad_numerator, grad_denominator, p, peers, s);
}


}  // namespace

// ---------------------------------------------------------------------------
// C ABI.
// ---------------------------------------------------------------------------

extern "C" {

const char* kat_rational_strerror(int status) {
  switch (status) {
    case KAT_OK: return "success";
    case KAT_ERR_NULL_POINTER: return "a required pointer argument is NULL";
    case KAT_ERR_BAD_DTYPE: return "unsupported dtype (expected KAT_DTYPE_F32, _F16 or _BF16)";
    case KAT_ERR_BAD_SHAPE: return "invalid shape: negative extent or size overflow";
    case KAT_ERR_BAD_GROUPS: return "num_groups must be >= 1 and divide channels";
    case KAT_ERR_WORKSPACE: return "workspace is NULL, misaligned or smaller than required";
    case KAT_ERR_CUDA: return "CUDA runtime or kernel launch error";
    case KAT_ERR_BAD_FORMULA:
      return "unsupported formula (expected KAT_FORMULA_KAT or KAT_FORMULA_ABS_SUM)";
    case KAT_ERR_SCRATCH_LIMIT:
      return "problem needs more backward scratch than kat_rational_bwd_noalloc's fixed "
             "2 MiB device buffer holds; use kat_rational_bwd with a caller-allocated workspace";
    default: return "unknown kat_rational status";
  }
}

int kat_rational_abi_version(void) { return KAT_RATIONAL_ABI_VERSION; }

int kat_rational_device_status(int device, int reset, int* status) {
  if (status == nullptr) return KAT_ERR_NULL_POINTER;
  int prev = 0;
  if (cudaGetDevice(&prev) != cudaSuccess) return KAT_ERR_CUDA;
  if (device != prev && cudaSetDevice(device) != cudaSuccess) return KAT_ERR_CUDA;
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_kat_status, sizeof(int));
  if (e == cudaSuccess && reset) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_kat_status, &zero, sizeof(int));
  }
  if (device != prev) cudaSetDevice(prev);
  if (e != cudaSuccess) return KAT_ERR_CUDA;
  *status = v;
  return KAT_OK;
}

int kat_rational_make_plan(int64_t batch, int64_t channels, int64_t inner, int64_t num_groups,
                           int dtype, int vec, int sm_count, int ctas_per_sm,
                           kat_rational_plan* plan) {
  if (plan == nullptr) return KAT_ERR_NULL_POINTER;
  Plan p;
  const int st = make_plan_impl(batch, channels, inner, num_groups, dtype, vec, sm_count,
                                ctas_per_sm, &p);
  if (st != KAT_OK) return st;
  to_public(p, plan);
  return KAT_OK;
}

}  // extern "C"

namespace {

// Float64 forward, for float64 tensors (gradient checking).  One element per thread in a
// grid-stride loop; the group of element i is ((i / inner) % channels) / (channels / G).
// Coefficients are float64 as well, and the arithmetic is float64 throughout (fma Horner,
// IEEE division), as the reference's Triton forward computes in its input dtype.
template <int kF>
__global__ void __launch_bounds__(256)
kat_fwd_f64_kernel(const double* __restrict__ x, double* __restrict__ y,
                   const double* __restrict__ num, const double* __restrict__ den, int64_t n,
                   int64_t inner, int64_t channels, int64_t per_group) {
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    const int64_t g = ((i / inner) % channels) / per_group;
    const double* a = num + g * 6;
    const double* b = den + g * 4;
    const double v = x[i];
    double p = fma(a[5], v, a[4]);
    p = fma(p, v, a[3]);
    p = fma(p, v, a[2]);
    p = fma(p, v, a[1]);
    p = fma(p, v, a[0]);
    double q;
    if constexpr (kF == kFormulaKat) {
      q = fma(fabs(b[3]), v, fabs(b[2]));
      q = fma(q, v, fabs(b[1]));
      q = fma(q, v, fabs(b[0]));
      q = fma(q, v, 1.0);
    } else {
      q = fma(b[3], v, b[2]);
      q = fma(q, v, b[1]);
      q = fma(q, v, b[0]);
      q = 1.0 + fabs(q * v);
    }
    y[i] = p / q;
  }
}

int fwd_f64_impl(const double* x, double* y, const double* numerator, const double* denominator,
                 int64_t batch, int64_t channels, int64_t inner, int64_t num_groups, int formula,
                 void* stream) {
  int64_t n = 0;
  int st = validate_dims(batch, channels, inner, num_groups, KAT_DTYPE_F32, &n);
  if (st != KAT_OK) return st;
  if (formula != kFormulaKat && formula != kFormulaAbsSum) return KAT_ERR_BAD_FORMULA;
  if (numerator == nullptr || denominator == nullptr) return KAT_ERR_NULL_POINTER;
  if (n == 0) return KAT_OK;
  if (x == nullptr || y == nullptr) return KAT_ERR_NULL_POINTER;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || device_sm_count(dev, &sms) != cudaSuccess)
    return KAT_ERR_CUDA;
  const int64_t blocks = std::min<int64_t>((n + 255) / 256, int64_t(sms) * 8);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t per_group = channels / num_groups;
  if (formula == kFormulaKat) {
    kat_fwd_f64_kernel<kFormulaKat><<<unsigned(blocks), 256, 0, s>>>(
        x, y, numerator, denominator, n, inner, channels, per_group);
  } else {
    kat_fwd_f64_kernel<kFormulaAbsSum><<<unsigned(blocks), 256, 0, s>>>(
        x, y, numerator, denominator, n, inner, channels, per_group);
  }
  return cudaGetLastError() == cudaSuccess ? KAT_OK : KAT_ERR_CUDA;
}

int fwd_impl(const void* x, void* y, const float* numerator, const float* denominator,
             int64_t batch, int64_t channels, int64_t inner, int64_t num_groups, int dtype,
             int formula, void* stream) {
  int64_t n = 0;
  int st = validate_dims(batch, channels, inner, num_groups, dtype, &n);
  if (st != KAT_OK) return st;
  const int num_stride = (formula & KAT_SHARED_NUMERATOR) ? 0 : 6;
  formula &= ~KAT_SHARED_NUMERATOR;
  if (formula != kFormulaKat && formula != kFormulaAbsSum) return KAT_ERR_BAD_FORMULA;
  if (numerator == nullptr || denominator == nullptr) return KAT_ERR_NULL_POINTER;
  if (n == 0) return KAT_OK;
  if (x == nullptr || y == nullptr) return KAT_ERR_NULL_POINTER;
  const int64_t gw = (channels / num_groups) * inner;
  const void* ptrs[2] = {x, y};
  const int vec = pick_vec(dtype, gw, ptrs, 2);
  Plan p;
  if (vec == max_vec_for(dtype) && formula == kFormulaKat) {
    Pipe q;
    int dev = 0;
    st = plan_tma(batch, channels, inner, num_groups, dtype, false, &dev, &p, &q);
    if (st != -1) {
      if (st != KAT_OK) return st;
      if (allow_dynamic_smem(dev, fwd_tma_kernel_for(dtype), q.smem_bytes) != cudaSuccess)
        return KAT_ERR_CUDA;
      p.num_stride = num_stride;
      if (launch_fwd_tma(dtype, x, y, numerator, denominator, p, q,
                         static_cast<cudaStream_t>(stream)) != cudaSuccess)
        return KAT_ERR_CUDA;
      return KAT_OK;
    }
  }
  st = plan_for_launch(fwd_kernel_for(dtype, vec, formula), batch, channels, inner, num_groups,
                       dtype, vec, &p);
  if (st != KAT_OK) return st;
  p.num_stride = num_stride;
  if (launch_fwd(dtype, vec, formula, x, y, numerator, denominator, p,
                 static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return KAT_ERR_CUDA;
  return KAT_OK;
}

}  // namespace

extern "C" {

int kat_rational_fwd(const void* x, void* y, const float* numerator, const float* denominator,
                     int64_t batch, int64_t channels, int64_t inner, int64_t num_groups, int dtype,
                     void* stream) {
  return fwd_impl(x, y, numerator, denominator, batch, channels, inner, num_groups, dtype,
                  kFormulaKat, stream);
}

int kat_rational_fwd_f64(const double* x, double* y, const double* numerator,
                         const double* denominator, int64_t batch, int64_t channels,
                         int64_t inner, int64_t num_groups, int formula, void* stream) {
  return fwd_f64_impl(x, y, numerator, denominator, batch, channels, inner, num_groups, formula,
                      stream);
}

int kat_rational_fwd_formula(const void* x, void* y, const float* numerator,
                             const float* denominator, int64_t batch, int64_t channels,
                             int64_t inner, int64_t num_groups, int dtype, int formula,
                             void* stream) {
  return fwd_impl(x, y, numerator, denominator, batch, channels, inner, num_groups, dtype,
                  formula, stream);
}

int kat_rational_bwd_workspace_size(int64_t batch, int64_t channels, int64_t inner,
                                    int64_t num_groups, int dtype, int device, size_t* bytes) {
  if (bytes == nullptr) return KAT_ERR_NULL_POINTER;
  int64_t n = 0;
  int st = validate_dims(batch, channels, inner, num_groups, dtype, &n);
  if (st != KAT_OK) return st;
  *bytes = 0;
  if (n == 0) return KAT_OK;
  int prev = 0;
  if (cudaGetDevice(&prev) != cudaSuccess) return KAT_ERR_CUDA;
  if (device != prev && cudaSetDevice(device) != cudaSuccess) return KAT_ERR_CUDA;
  const int64_t gw = (channels / num_groups) * inner;
  uint64_t need = 0;
  {
    Plan p;
    Pipe q;
    int d = 0;
    const int t = plan_tma(batch, channels, inner, num_groups, dtype, true, &d, &p, &q);
    if (t == KAT_OK) need = p.workspace_bytes;
    else if (t != -1) st = t;
    const int vecs[2] = {max_vec_for(dtype), 8 / elem_bytes(dtype)};
    for (int v : vecs) {
      for (int f = kFormulaKat; st == KAT_OK && f <= kFormulaAbsSum; ++f) {
        if (gw % v != 0) continue;
        const int a = plan_async(batch, channels, inner, num_groups, dtype, f, &d, &p, v);
        if (a == KAT_OK) need = std::max<uint64_t>(need, p.workspace_bytes);
        else if (a != -1) st = a;
      }
    }
  }
  // Enough for every kernel the backward may pick, for either formula.
  for (int vec = max_vec_for(dtype); st == KAT_OK && vec >= 1; vec >>= 1) {
    if (gw % vec != 0) continue;
    for (int f = kFormulaKat; st == KAT_OK && f <= kFormulaAbsSum; ++f) {
      Plan p;
      st = plan_for_launch(bwd_kernel_for(dtype, vec, f), batch, channels, inner, num_groups,
                           dtype, vec, &p);
      if (st == KAT_OK && p.workspace_bytes > need) need = p.workspace_bytes;
    }
  }
  if (device != prev) cudaSetDevice(prev);
  if (st != KAT_OK) return st;
  *bytes = size_t(need);
  return KAT_OK;
}

int kat_rational_bwd(const void* x, const void* grad_out, void* grad_x, const float* numerator,
                     const float* denominator, float* grad_numerator, float* grad_denominator,
                     void* workspace, size_t workspace_bytes, int64_t batch, int64_t channels,
                     int64_t inner, int64_t num_groups, int dtype, void* stream) {
  return bwd_impl(x, grad_out, grad_x, numerator, denominator, grad_numerator, grad_denominator,
                  workspace, workspace_bytes, batch, channels, inner, num_groups, dtype,
                  kFormulaKat, stream, nullptr);
}

int kat_rational_bwd_formula(const void* x, const void* grad_out, void* grad_x,
                             const float* numerator, const float* denominator,
                             float* grad_numerator, float* grad_denominator, void* workspace,
                             size_t workspace_bytes, int64_t batch, int64_t channels,
                             int64_t inner, int64_t num_groups, int dtype, int formula,
                             void* stream) {
  return bwd_impl(x, grad_out, grad_x, numerator, denominator, grad_numerator, grad_denominator,
                  workspace, workspace_bytes, batch, channels, inner, num_groups, dtype, formula,
                  stream, nullptr);
}

int kat_rational_enable_peer_access(int device, int peer_device) {
  if (device == peer_device) return KAT_OK;
  int prev = 0;
  if (cudaGetDevice(&prev) != cudaSuccess) return KAT_ERR_CUDA;
  if (cudaSetDevice(device) != cudaSuccess) return KAT_ERR_CUDA;
  int can = 0;
  cudaError_t e = cudaDeviceCanAccessPeer(&can, device, peer_device);
  if (e == cudaSuccess && can) {
    e = cudaDeviceEnablePeerAccess(peer_device, 0);
    if (e == cudaErrorPeerAccessAlreadyEnabled) {
      cudaGetLastError();
      e = cudaSuccess;
    }
  } else if (e == cudaSuccess) {
    e = cudaErrorPeerAccessUnsupported;
  }
  cudaSetDevice(prev);
  return e == cudaSuccess ? KAT_OK : KAT_ERR_CUDA;
}

// Exchange buffers (setup-time plumbing, outside the per-step path).  The local buffer is
// allocated here so that its CUDA IPC handle covers exactly it; peers' handles are opened
// with this process's current device current and lazy peer access, so the mapping is usable
// by kernels on that device.
int kat_rational_exchange_create(int64_t num_groups, void** buffer, void* ipc_handle) {
  if (buffer == nullptr || ipc_handle == nullptr) return KAT_ERR_NULL_POINTER;
  if (num_groups < 1) return KAT_ERR_BAD_GROUPS;
  const size_t bytes = kExchangeHeader + size_t(2) * kMaxPeers * size_t(num_groups) * kAcc * 16;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return KAT_ERR_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return KAT_ERR_CUDA;
  }
  memcpy(ipc_handle, &h, sizeof(h));
  *buffer = p;
  return KAT_OK;
}

int kat_rational_exchange_open(const void* ipc_handle, void* local_probe, void** peer_buffer) {
  if (ipc_handle == nullptr || peer_buffer == nullptr || local_probe == nullptr)
    return KAT_ERR_NULL_POINTER;
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
    return KAT_ERR_CUDA;
  // Prove the mapping is reachable from this device before any kernel may touch it.
  cudaPointerAttributes attr;
  if (cudaPointerGetAttributes(&attr, p) != cudaSuccess || attr.type != cudaMemoryTypeDevice ||
      cudaMemcpy(local_probe, p, 16, cudaMemcpyDeviceToDevice) != cudaSuccess) {
    cudaGetLastError();
    cudaIpcCloseMemHandle(p);
    return KAT_ERR_CUDA;
  }
  *peer_buffer = p;
  return KAT_OK;
}

int kat_rational_exchange_close(void* peer_buffer) {
  return cudaIpcCloseMemHandle(peer_buffer) == cudaSuccess ? KAT_OK : KAT_ERR_CUDA;
}

int kat_rational_exchange_destroy(void* buffer) {
  return cudaFree(buffer) == cudaSuccess ? KAT_OK : KAT_ERR_CUDA;
}

size_t kat_rational_exchange_buffer_bytes(int64_t num_groups) {
  if (num_groups < 1) return 0;
  return kExchangeHeader + size_t(2) * kMaxPeers * size_t(num_groups) * kAcc * 16;
}

}  // extern "C"

namespace {

// Checks a kat_rational_peers descriptor and copies it into the kernels' form.
int peers_from(const kat_rational_peers* peers, int64_t num_groups, Peers* pe) {
  if (peers == nullptr) return KAT_ERR_NULL_POINTER;
  if (peers->world_size < 1 || peers->world_size > KAT_MAX_PEERS || peers->rank < 0 ||
      peers->rank >= peers->world_size || peers->timeout_ms < 1)
    return KAT_ERR_BAD_SHAPE;
  if (num_groups < 1 || num_groups * kAcc * int64_t(sizeof(double)) > 200 * 1024)
    return KAT_ERR_BAD_GROUPS;
  memset(pe, 0, sizeof(*pe));
  pe->world = peers->world_size;
  pe->rank = peers->rank;
  pe->average = peers->average ? 1 : 0;
  pe->timeout_ms = peers->timeout_ms;
  for (int r = 0; r < pe->world; ++r) {
    if (peers->buffers[r] == nullptr || (reinterpret_cast<uintptr_t>(peers->buffers[r]) % 16) != 0)
      return KAT_ERR_NULL_POINTER;
    pe->buf[r] = static_cast<char*>(peers->buffers[r]);
  }
  return KAT_OK;
}

}  // namespace

extern "C" {

int kat_rational_bwd_allreduce(const void* x, const void* grad_out, void* grad_x,
                               const float* numerator, const float* denominator,
                               float* grad_numerator, float* grad_denominator, void* workspace,
                               size_t workspace_bytes, int64_t batch, int64_t channels,
                               int64_t inner, int64_t num_groups, int dtype,
                               const kat_rational_peers* peers, void* stream) {
  Peers pe;
  const int st = peers_from(peers, num_groups, &pe);
  if (st != KAT_OK) return st;
  return bwd_impl(x, grad_out, grad_x, numerator, denominator, grad_numerator, grad_denominator,
                  workspace, workspace_bytes, batch, channels, inner, num_groups, dtype,
                  kFormulaKat, stream, &pe);
}

int kat_rational_bwd_allreduce_formula(const void* x, const void* grad_out, void* grad_x,
                                       const float* numerator, const float* denominator,
                                       float* grad_numerator, float* grad_denominator,
                                       void* workspace, size_t workspace_bytes, int64_t batch,
                                       int64_t channels, int64_t inner, int64_t num_groups,
                                       int dtype, int formula, const kat_rational_peers* peers,
                                       void* stream) {
  if ((formula & ~KAT_SHARED_NUMERATOR) != kFormulaKat) return KAT_ERR_BAD_FORMULA;
  Peers pe;
  const int st = peers_from(peers, num_groups, &pe);
  if (st != KAT_OK) return st;
  return bwd_impl(x, grad_out, grad_x, numerator, denominator, grad_numerator, grad_denominator,
                  workspace, workspace_bytes, batch, channels, inner, num_groups, dtype,
                  formula, stream, &pe);
}

int kat_rational_exchange_grads(float* grad_numerator, float* grad_denominator,
                                int64_t num_groups, const kat_rational_peers* peers,
                                void* stream) {
  if (grad_numerator == nullptr || grad_denominator == nullptr) return KAT_ERR_NULL_POINTER;
  Peers pe;
  const int st = peers_from(peers, num_groups, &pe);
  if (st != KAT_OK) return st;
  const size_t smem = size_t(num_groups) * kAcc * sizeof(double);
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute((const void*)kat_exchange_grads_kernel,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess)
    return KAT_ERR_CUDA;
  kat_exchange_grads_kernel<<<1, kReduceThreads, smem, static_cast<cudaStream_t>(stream)>>>(
      grad_numerator, grad_denominator, int(num_groups), pe);
  return cudaGetLastError() == cudaSuccess ? KAT_OK : KAT_ERR_CUDA;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Backward without allocation.
//
// kat_rational_bwd needs a caller-allocated workspace for its per-block partial sums.  Some
// callers cannot allocate device memory where they run the backward: plugin hosts whose
// operator interface hands over input/output buffers but no allocator, and fixed-budget
// real-time loops where a cudaMalloc in the middle of a run may stall the device or fail.
// For them, kat_rational_bwd_noalloc uses a fixed file-scope device array as that workspace.
// ---------------------------------------------------------------------------

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(2) << 20;  // 2 MiB on every device in use

// The workspace of kat_rational_bwd_noalloc.  In host code this name only stands in for
// the device symbol; its device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) double g_noalloc_scratch[kNoAllocScratchBytes / sizeof(double)];

std::mutex g_noalloc_mu;
std::map<int, void*> g_noalloc_addr;

// Device address of the scratch array on `dev`, which must be the current device; looked up
// once per device and cached for the life of the process (the address of the device's
// primary context at the first call: a cudaDeviceReset afterwards leaves it stale).
cudaError_t noalloc_scratch_address(int dev, void** out) {
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  auto it = g_noalloc_addr.find(dev);
  if (it != g_noalloc_addr.end()) {
    *out = it->second;
    return cudaSuccess;
  }
  void* ptr = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
  if (e != cudaSuccess) return e;
  g_noalloc_addr[dev] = ptr;
  *out = ptr;
  return cudaSuccess;
}

}  // namespace

extern "C" int kat_rational_bwd_noalloc(const void* x, const void* grad_out, void* grad_x,
                                        const float* numerator, const float* denominator,
                                        float* grad_numerator, float* grad_denominator,
                                        int64_t batch, int64_t channels, int64_t inner,
                                        int64_t num_groups, int dtype, void* stream) {
  int64_t n = 0;
  int st = validate_dims(batch, channels, inner, num_groups, dtype, &n);
  if (st != KAT_OK) return st;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return KAT_ERR_CUDA;
  size_t need = 0;
  st = kat_rational_bwd_workspace_size(batch, channels, inner, num_groups, dtype, dev, &need);
  if (st != KAT_OK) return st;
  if (need > kNoAllocScratchBytes) return KAT_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  if (noalloc_scratch_address(dev, &scratch) != cudaSuccess) return KAT_ERR_CUDA;
  return kat_rational_bwd(x, grad_out, grad_x, numerator, denominator, grad_numerator,
                          grad_denominator, scratch, kNoAllocScratchBytes, batch, channels, inner,
                          num_groups, dtype, stream);
}
