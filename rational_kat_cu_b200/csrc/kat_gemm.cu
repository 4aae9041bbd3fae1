// kat_gemm.cu — sm_100a tensor-core GEMM (C = A B^T, bf16 in, fp32 accumulate) with the
// group-rational activation fused into its epilogue (C ABI: include/kat_gemm.h).
//
// One persistent CTA per SM (or one CTA pair per two SMs, below), three roles:
//   warp 0, one lane   TMA producer: per k-block, a 128 x 64 tile of A and a 256 x 64 tile of B
//                      (bf16, 128-byte swizzled rows) into a ring of shared-memory stages;
//   warp 1, one lane   MMA issuer: tcgen05.mma (kind::f16, M = 128, N = 256, K = 16) from the
//                      stage's shared-memory descriptors into one of two 256-column fp32
//                      accumulators in tensor memory; tcgen05.commit frees the stage when its
//                      MMAs have read it and, after the last k-block, hands the accumulator to
//                      the epilogue.  Warp 1 also allocates and frees the 512 TMEM columns;
//   warps 2 ..         epilogue, independent warps (8 for the plain and forward epilogues, 16
//                      for the FP32-heavy backward): warp w owns the 32 accumulator rows of its
//                      TMEM lane quadrant (a warp may read only lanes 32 (w % 4) .. + 31) and
//                      one column slice of the tile, which it reads 16 columns at a time with
//                      tcgen05.ld (the next load in flight while the previous half is
//                      computed), runs through the epilogue, writes as bf16 into its own
//                      64-byte-swizzled 32 x 32 staging tile and stores with TMA (lane 0).
// With two accumulators the epilogue of one output tile overlaps the mainloop of the next.
// Tiles are numbered column-block-major and every CTA (pair) takes one contiguous run of them,
// so a CTA's tiles mostly share one 256-column block of B and one set of channel groups (few
// coefficient reloads and gradient flushes); A and B are re-read from L2.
//
// CTA pairs (cta_group::2, a 2-CTA cluster per 256 x 256 tile): each CTA loads its 128 rows
// of A and its half of B's rows, both CTAs' TMA loads count on the rank-0 CTA's barrier, the
// rank-0 CTA issues M = 256 MMAs and commits to the barriers of both CTAs, each CTA's epilogue
// reads its own 128 accumulator rows.  Used when 256-row tiles take no more waves than 128-row
// tiles.
//
// Epilogues: plain (C = bf16(acc + bias)); forward (h = bf16(acc + bias), y = rational(h) with
// the activation kernels' per-element math, so y is bit-identical to kat_rational_fwd on h);
// backward (g = bf16(acc), the warp's 32 x 32 tile of h loaded by TMA one chunk ahead, dh = the
// activation kernels' per-element backward on (h, g), per-thread fp32 gradient sums flushed in
// a fixed order into per-warp fp64 partials, summed per CTA in warp order at the end, then a
// second kernel adds the CTA sums in a fixed order).
//
// Every mbarrier wait is bounded (about two seconds of clock cycles).  A wait that runs out
// sets the CTA's abort flag and the sticky device status word; the other roles see the flag
// in their own waits and stop, the MMA issuer drains its outstanding MMAs and warp 1 frees the
// tensor memory before the CTA exits.

#include <cuda.h>  // CUtensorMap and its enums (types only: the encoder is fetched at run time)
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <mutex>

#include "kat_rational.h"
#include "kat_gemm.h"

namespace {

#include "kat_math.cuh"

constexpr int kBM = 128;       // tile rows (MMA M, TMEM lanes)
constexpr int kBN = 256;       // tile columns (MMA N, TMEM columns per accumulator)
constexpr int kBK = 64;        // k-block: 64 bf16 = one 128-byte swizzle row
constexpr int kUmmaK = 16;     // K of one kind::f16 MMA
constexpr int kEpiWarp0 = 2;
constexpr int kMaxEpiWarps = 16;
constexpr int kChunk = 32;                     // columns per staging tile / TMA store
constexpr int kHalf = 16;                      // columns per tcgen05.ld
constexpr int kWarpRows = 32;
constexpr uint32_t kTmemCols = 2 * kBN;
constexpr uint32_t kABytes = kBM * kBK * 2;
constexpr uint32_t kTileBytes = kWarpRows * kChunk * 2;  // 32 rows x 64 bytes
constexpr uint32_t kBarBytes = 512;
constexpr long long kWaitCycles = 4000000000LL;
constexpr int kStatusWaitTimeout = KAT_DEVICE_WAIT_TIMEOUT;

enum Mode { kPlain = 0, kFwd = 1, kBwd = 2 };

// Per mode: mainloop stages (one CTA per tile / two CTAs per 256-row tile), epilogue warps (a
// multiple of 4: one per TMEM lane quadrant and column slice), staging tiles per epilogue warp
// (outputs) and h tiles per epilogue warp.  The light plain / forward epilogues keep up with 8
// warps; the FP32-heavy backward epilogue gets 16 warps (4 per SM sub-partition).
template <int kMode> struct Cfg;
template <> struct Cfg<kPlain> {
  static constexpr int kStages1 = 4, kStages2 = 6, kEpiWarps = 8, kOuts = 1, kH = 0;
};
template <> struct Cfg<kFwd> {
  static constexpr int kStages1 = 4, kStages2 = 6, kEpiWarps = 8, kOuts = 2, kH = 0;
};
template <> struct Cfg<kBwd> {
  static constexpr int kStages1 = 3, kStages2 = 4, kEpiWarps = 16, kOuts = 1, kH = 1;
};

template <int kMode, int kPair>
__host__ __device__ constexpr int stages_of() {
  return kPair == 2 ? Cfg<kMode>::kStages2 : Cfg<kMode>::kStages1;
}
// With two CTAs per tile each CTA holds half of B's 256 rows (the MMA reads both halves).
template <int kPair>
__host__ __device__ constexpr uint32_t b_bytes() {
  return uint32_t(kBN / kPair) * kBK * 2;
}

template <int kMode>
__host__ __device__ constexpr int threads_of() {
  return (kEpiWarp0 + Cfg<kMode>::kEpiWarps) * 32;
}

template <int kMode, int kPair>
__host__ __device__ constexpr uint32_t smem_bytes() {
  return 1024 + stages_of<kMode, kPair>() * (kABytes + b_bytes<kPair>()) +
         Cfg<kMode>::kEpiWarps * (Cfg<kMode>::kOuts + Cfg<kMode>::kH) * kTileBytes + kBarBytes;
}
static_assert(smem_bytes<kPlain, 1>() <= 227 * 1024, "plain shared memory");
static_assert(smem_bytes<kFwd, 1>() <= 227 * 1024, "forward shared memory");
static_assert(smem_bytes<kBwd, 1>() <= 227 * 1024, "backward shared memory");
static_assert(smem_bytes<kPlain, 2>() <= 227 * 1024, "plain shared memory (pairs)");
static_assert(smem_bytes<kFwd, 2>() <= 227 * 1024, "forward shared memory (pairs)");
static_assert(smem_bytes<kBwd, 2>() <= 227 * 1024, "backward shared memory (pairs)");

struct GemmArgs {
  int32_t m;            // rows of A and of the outputs
  int32_t m_tiles;      // row tiles (ceil(M / (128 x CTAs per tile)))
  int32_t n_tiles;      // column tiles (N / 256)
  int32_t num_tiles;    // row tiles x column tiles
  int32_t k_blocks;     // K / 64
  int32_t group_width;  // N / G (multiple of 32)
  int32_t groups;
  const uint16_t* bias;   // bf16 [N] or null
  const float* num;       // [G, 6]
  const float* den;       // [G, 4]
  double* partial;        // backward: [grid][16 warps][G][10]; row 0 of a CTA ends as its sum
  int32_t stall;          // test hook: the MMA issuer waits on a barrier nothing completes
  int32_t store_h;        // forward: 0 = y only (inference), h is neither staged nor stored
};

__device__ int g_gemm_status;

// ---------------------------------------------------------------------------
// PTX wrappers.
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}
// try_wait that lets the thread sleep in hardware until the phase completes or about
// kSuspendNs have passed, so a waiting thread takes no issue slots from the busy warps.
constexpr uint32_t kSuspendNs = 20000;
__device__ __forceinline__ bool mbar_try_suspend(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendNs)
      : "memory");
  return done != 0;
}
// Bounded wait of one thread for the phase with `parity`; false when the CTA aborted or this
// wait ran out (which aborts the CTA).
__device__ __forceinline__ bool wait_phase(uint64_t* bar, uint32_t parity, volatile int* abort) {
  if (mbar_try(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_suspend(bar, parity)) {
    if (*abort) return false;
    if (clock64() - t0 > kWaitCycles) {
      *abort = 1;
      atomicExch(&g_gemm_status, kStatusWaitTimeout);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int32_t x,
                                             int32_t y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
template <int kPending>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(kPending) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void fence_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Tensor memory, MMA and commit for one CTA (kPair = 1) or a CTA pair of a cluster (kPair = 2:
// issued by the pair's rank-0 CTA, operands and accumulator split across both CTAs).
template <int kPair>
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t cols) {
  if constexpr (kPair == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(slot)), "r"(cols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  } else {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(slot)), "r"(cols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
}
template <int kPair>
__device__ __forceinline__ void tmem_free(uint32_t base, uint32_t cols) {
  if constexpr (kPair == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(cols)
                 : "memory");
  } else {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(cols)
                 : "memory");
  }
}
// D[tmem] (+)= A[smem] B[smem]^T for one K = 16 slice.
template <int kPair>
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  if constexpr (kPair == 1) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  }
}
// Arrive once on the mbarrier at shared::cluster address `bar` (this CTA's or the pair peer's)
// when every MMA this thread issued so far has completed.
template <int kPair>
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  if constexpr (kPair == 1) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     bar) : "memory");
  } else {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     bar) : "memory");
  }
}
// shared::cluster address of the object at `p` in the cluster's CTA `rank`.
__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" :::
                   "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar)
               : "memory");
}
// TMA load into this CTA's shared memory whose completion is counted on the pair's rank-0
// barrier `bar` (a shared::cluster address).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar,
                                                 int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
// 16 consecutive fp32 columns of this thread's TMEM lane; the values are valid after
// tmem_wait on the same registers.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32"
      " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),
        "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr)
      : "memory");
}
// Wait for this thread's outstanding tcgen05.ld; the registers are tied to the wait so no use
// of them is scheduled before it.
__device__ __forceinline__ void tmem_wait(uint32_t (&v)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]),
                 "+r"(v[6]), "+r"(v[7]), "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]),
                 "+r"(v[12]), "+r"(v[13]), "+r"(v[14]), "+r"(v[15])
               :
               : "memory");
}

// Shared-memory matrix descriptor of a K-major bf16 tile with 128-byte rows, 128-byte swizzle,
// 8-row groups 1024 bytes apart (tcgen05 descriptor: start >> 4 in bits 0-13, leading byte
// offset 16 >> 4 in 16-29 (unused by swizzled K-major layouts), stride byte offset 1024 >> 4 in
// 32-45, descriptor version 1 in 46-47, swizzle mode 2 = 128B in 61-63).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return uint64_t((saddr & 0x3FFFFu) >> 4) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) |
         (uint64_t(1) << 46) | (uint64_t(2) << 61);
}
// Instruction descriptor: fp32 accumulator (bits 4-5 = 1), A and B bf16 (7-9 = 1, 10-12 = 1),
// both K-major (15, 16 = 0), N >> 3 in 17-22, M >> 4 in 24-28 (M = 256 for a CTA pair).
template <int kPair>
__host__ __device__ constexpr uint32_t idesc_of() {
  return (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(kBN >> 3) << 17) |
         (uint32_t((kBM * kPair) >> 4) << 24);
}

// Byte offset of 16-byte granule j (0..3) of row r in a 64-byte-swizzled tile (the TMA
// SWIZZLE_64B pattern: granule index XOR address bits 7-8).
__device__ __forceinline__ uint32_t sw64_offset(int r, int j) {
  return uint32_t(r) * 64u + uint32_t((j ^ ((r >> 1) & 3)) << 4);
}

__device__ __forceinline__ float bf16_bits_to_float(uint32_t bits16) {
  return __uint_as_float(bits16 << 16);
}

// ---------------------------------------------------------------------------
// The kernel.
// ---------------------------------------------------------------------------

template <int kMode, int kF, int kPair>
__global__ void __launch_bounds__(threads_of<kMode>(), 1)
kat_gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                const __grid_constant__ CUtensorMap tm_out0,
                const __grid_constant__ CUtensorMap tm_out1,
                const __grid_constant__ CUtensorMap tm_h, const GemmArgs args) {
  constexpr int S = stages_of<kMode, kPair>();
  constexpr uint32_t kBBytes = b_bytes<kPair>();
  constexpr int kOuts = Cfg<kMode>::kOuts;
  constexpr int kEpiWarps = Cfg<kMode>::kEpiWarps;
  constexpr int kSlice = kBN / (kEpiWarps / 4);  // columns per epilogue warp and tile
  constexpr int kChunksPerSlice = kSlice / kChunk;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* s_a = smem;
  uint8_t* s_b = s_a + S * kABytes;
  uint8_t* s_out = s_b + S * kBBytes;                  // [epilogue warp][kOuts] 32 x 32 tiles
  uint8_t* s_h = s_out + kEpiWarps * kOuts * kTileBytes;  // backward: [epilogue warp] h tile
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_h + kEpiWarps * Cfg<kMode>::kH * kTileBytes);
  uint64_t* full = bars;              // [S]  TMA -> MMA (rank 0's counts both CTAs' bytes)
  uint64_t* empty = full + S;         // [S]  MMA -> TMA (in each CTA)
  uint64_t* tfull = empty + S;        // [2]  MMA -> epilogue (in each CTA)
  uint64_t* tempty = tfull + 2;       // [2]  epilogue warps of both CTAs -> MMA (rank 0's)
  uint64_t* hbar = tempty + 2;        // [kEpiWarps] backward h loads
  uint64_t* drain = hbar + kEpiWarps; // MMA completion before teardown
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = kPair == 2 ? cluster_rank() : 0u;   // position in the CTA pair
  const int slot0 = int(blockIdx.x) / kPair;                 // tile slot of this CTA (pair)
  const int slots = int(gridDim.x) / kPair;
  // Each slot takes one contiguous run of the column-block-major tile order (an even split),
  // so its tiles mostly share one 256-column block and one set of channel groups.
  const int tile_begin = int(int64_t(slot0) * args.num_tiles / slots);
  const int tile_end = int(int64_t(slot0 + 1) * args.num_tiles / slots);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int j = 0; j < 2; ++j) {
      mbar_init(tfull + j, 1);
      mbar_init(tempty + j, kPair * kEpiWarps);
    }
    for (int j = 0; j < kEpiWarps; ++j) mbar_init(hbar + j, 1);
    mbar_init(drain, 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    prefetch_map(&tm_a);
    prefetch_map(&tm_b);
    prefetch_map(&tm_out0);
    if (kMode == kFwd) prefetch_map(&tm_out1);
    if (kMode == kBwd) prefetch_map(&tm_h);
  }
  if (warp == 1) tmem_alloc<kPair>(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  if constexpr (kPair == 2) cluster_sync();  // the peer's barriers exist before any remote use
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int m_tiles = args.m_tiles;
  const int k_blocks = args.k_blocks;

  if (warp == 0) {
    // ---------------- TMA producer (each CTA loads its A rows and its half of B) ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = tile_begin; tile < tile_end; ++tile) {
        const int m0 = (tile % m_tiles) * (kBM * kPair) + int(rank) * kBM;
        const int n0 = (tile / m_tiles) * kBN + int(rank) * (kBN / kPair);
        bool ok = true;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!wait_phase(empty + stage, phase ^ 1u, abort)) { ok = false; break; }
          if constexpr (kPair == 1) {
            mbar_expect_tx(full + stage, kABytes + kBBytes);
            tma_load_2d(s_a + stage * kABytes, &tm_a, full + stage, kb * kBK, m0);
            tma_load_2d(s_b + stage * kBBytes, &tm_b, full + stage, kb * kBK, n0);
          } else {
            if (rank == 0) mbar_expect_tx(full + stage, 2 * (kABytes + kBBytes));
            const uint32_t bar0 = cluster_addr(full + stage, 0);
            tma_load_2d_pair(s_a + stage * kABytes, &tm_a, bar0, kb * kBK, m0);
            tma_load_2d_pair(s_b + stage * kBBytes, &tm_b, bar0, kb * kBK, n0);
          }
          if (++stage == S) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (rank 0 of a pair issues for both CTAs) ----------------
    if (lane == 0 && rank == 0 && args.stall) {
      // Test hook (kat_gemm_set_test_stall): a wait that nothing completes runs out, sets the
      // abort flag and the device status, and every role stops at its next wait.
      (void)wait_phase(drain, 0u, abort);
    } else if (lane == 0 && rank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool issued = false;
      // arrive on the barrier in this CTA and, for a pair, on the same barrier in the peer
      auto commit_both = [&](uint64_t* bar) {
        umma_commit<kPair>(cluster_addr(bar, 0));
        if constexpr (kPair == 2) umma_commit<kPair>(cluster_addr(bar, 1));
      };
      for (int tile = tile_begin; tile < tile_end; ++tile, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!wait_phase(tempty + acc, acc_phase ^ 1u, abort)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t(acc * kBN);
        bool ok = true;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!wait_phase(full + stage, phase, abort)) { ok = false; break; }
          tc_fence_after();
          const uint64_t a_desc = sw128_desc(smem_u32(s_a + stage * kABytes));
          const uint64_t b_desc = sw128_desc(smem_u32(s_b + stage * kBBytes));
#pragma unroll
          for (int k = 0; k < kBK / kUmmaK; ++k) {
            // advance the start address by k x 32 bytes inside the swizzled 128-byte rows
            umma_bf16<kPair>(d_tmem, a_desc + uint64_t(k * 2), b_desc + uint64_t(k * 2),
                             idesc_of<kPair>(), (kb | k) != 0 ? 1u : 0u);
          }
          issued = true;
          commit_both(empty + stage);
          if (++stage == S) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        commit_both(tfull + acc);
      }
      if (issued) {
        // Every MMA has completed before the tensor memory is freed (bounded by the clock
        // alone: on the normal path this returns at once).
        umma_commit<kPair>(cluster_addr(drain, 0));
        const long long t0 = clock64();
        while (!mbar_try(drain, 0)) {
          if (clock64() - t0 > kWaitCycles) {
            atomicExch(&g_gemm_status, kStatusWaitTimeout);
            break;
          }
        }
      }
    }
  } else {
    // ---------------- epilogue (independent warps) ----------------
    const int ew = warp - kEpiWarp0;              // 0 .. kEpiWarps - 1
    const int quad = warp & 3;                    // TMEM lane quadrant this warp may access
    const int slice = ew >> 2;                    // 64-column slice of the tile
    const int row = lane;                         // row within the warp's 32-row tile
    const uint32_t lane_addr = tmem_base + (uint32_t(quad * 32) << 16);
    uint8_t* stage_out = s_out + ew * kOuts * kTileBytes;
    uint8_t* stage_h = s_h + ew * kTileBytes;
    uint64_t* my_hbar = hbar + ew;

    double* wpart = nullptr;
    if constexpr (kMode == kBwd) {
      wpart = args.partial + (size_t(blockIdx.x) * kEpiWarps + ew) * size_t(args.groups) * kAcc;
      for (int i = lane; i < args.groups * kAcc; i += 32) wpart[i] = 0.0;
      __syncwarp();
    }
    // A tile's origin for this warp: rows quad * 32 .. + 31 of this CTA's 128 rows, columns
    // slice * kSlice .. + kSlice - 1 (chunk c starts kChunk * c further).  Computed once per tile.
    auto tile_origin = [&](int tile, int& m0, int& n_base) {
      const int tm = tile % m_tiles;
      const int tn = tile / m_tiles;
      m0 = tm * (kBM * kPair) + int(rank) * kBM + quad * kWarpRows;
      n_base = tn * kBN + slice * kSlice;
    };
    auto issue_h = [&](int m0, int n0) {
      if constexpr (kMode == kBwd) {
        mbar_expect_tx(my_hbar, kTileBytes);
        tma_load_2d(stage_h, &tm_h, my_hbar, n0, m0);
      }
    };
    if (kMode == kBwd && lane == 0 && tile_begin < tile_end) {
      int m0, nb;
      tile_origin(tile_begin, m0, nb);
      issue_h(m0, nb);
    }

    FwdCoef<float2> fc;
    BwdCoef<float2> bc;
    float2 acc_g[kAcc];
#pragma unroll
    for (int k = 0; k < kAcc; ++k) acc_g[k] = make_float2(0.0f, 0.0f);
    int cur_group = -1;

    // Fixed-order flush of this warp's gradient sums for `g` into its fp64 partial row.
    auto flush = [&](int g) {
      double tot[kAcc];
#pragma unroll
      for (int k = 0; k < kAcc; ++k) {
        double v = double(acc_g[k].x) + double(acc_g[k].y);
#pragma unroll
        for (int m = 16; m > 0; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
        tot[k] = v;
        acc_g[k] = make_float2(0.0f, 0.0f);
      }
      double mine = 0.0;
#pragma unroll
      for (int k = 0; k < kAcc; ++k)
        if (lane == k) mine = tot[k];
      if (lane < kAcc) wpart[size_t(g) * kAcc + lane] += mine;
    };
    // Lane 0 waits (bounded); the warp leaves together on the broadcast outcome.
    auto warp_wait = [&](uint64_t* bar, uint32_t parity) -> bool {
      int ok = 1;
      if (lane == 0) ok = wait_phase(bar, parity, abort) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (ok) (void)mbar_try(bar, parity);  // completed: acquire for every lane
      return ok != 0;
    };

    int q = 0;
    int local = 0;
    bool alive = true;
    const uint32_t tempty0 = cluster_addr(tempty, 0);  // rank 0's tempty[0]
    for (int tile = tile_begin; tile < tile_end && alive; ++tile, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      int m0, n_base;
      tile_origin(tile, m0, n_base);
      if (!warp_wait(tfull + acc, acc_phase)) break;
      tc_fence_after();
      for (int c = 0; c < kChunksPerSlice; ++c, ++q) {
        const int n0 = n_base + c * kChunk;
        const int g = n0 / args.group_width;
        uint32_t hw[16];
        if constexpr (kMode == kBwd) {
          if (!warp_wait(my_hbar, uint32_t(q & 1))) { alive = false; break; }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint4 u = *reinterpret_cast<const uint4*>(stage_h + sw64_offset(row, j));
            hw[j * 4 + 0] = u.x; hw[j * 4 + 1] = u.y; hw[j * 4 + 2] = u.z; hw[j * 4 + 3] = u.w;
          }
          __syncwarp();  // the h tile is in registers: load the next chunk's into it
          if (lane == 0) {
            if (c + 1 < kChunksPerSlice) {
              issue_h(m0, n0 + kChunk);
            } else if (tile + 1 < tile_end) {
              int nm0, nnb;
              tile_origin(tile + 1, nm0, nnb);
              issue_h(nm0, nnb);
            }
          }
          if (g != cur_group) {
            if (cur_group >= 0) flush(cur_group);
            cur_group = g;
            load_bwd_coef<float2, kF>(args.num, args.den, g, bc);
          }
        } else if constexpr (kMode == kFwd) {
          if (g != cur_group) {
            cur_group = g;
            load_fwd_coef<float2, kF>(args.num, args.den, g, fc);
          }
        }
        // The chunk's 32 bias values (zeros without a bias), loaded before the accumulator so
        // their latency overlaps the TMEM loads.
        uint4 bias_words[4];
        if constexpr (kMode == kPlain || kMode == kFwd) {
          if (args.bias != nullptr) {
            const uint4* bp = reinterpret_cast<const uint4*>(args.bias + n0);
#pragma unroll
            for (int j = 0; j < 4; ++j) bias_words[j] = __ldg(bp + j);
          } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) bias_words[j] = make_uint4(0u, 0u, 0u, 0u);
          }
        }
        // One 16-column half: epilogue math on v, bf16 words into the staging tile(s).
        auto do_half = [&](uint32_t (&v)[16], const int half) {
          uint32_t w0[8];
          uint32_t w1[8];
          if constexpr (kMode == kPlain || kMode == kFwd) {
            float bias[16];
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              const uint4 u = bias_words[half * 2 + j];
              const uint32_t uw[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
              for (int t = 0; t < 4; ++t) {
                bias[j * 8 + t * 2] = bf16_bits_to_float(uw[t] & 0xFFFFu);
                bias[j * 8 + t * 2 + 1] = bf16_bits_to_float(uw[t] >> 16);
              }
            }
#pragma unroll
            for (int p = 0; p < 8; ++p) {
              const float2 hv =
                  make_float2(__fadd_rn(__uint_as_float(v[2 * p]), bias[2 * p]),
                              __fadd_rn(__uint_as_float(v[2 * p + 1]), bias[2 * p + 1]));
              w0[p] = Codec<__nv_bfloat16>::pack_word(hv);
              if constexpr (kMode == kFwd) {
                const float2 hx = Codec<__nv_bfloat16>::unpack_word(w0[p]);
                w1[p] = Codec<__nv_bfloat16>::pack_word(fwd_math<float2, false, kF>(hx, fc));
              }
            }
          } else {
#pragma unroll
            for (int p = 0; p < 8; ++p) {
              const uint32_t gw = Codec<__nv_bfloat16>::pack_word(
                  make_float2(__uint_as_float(v[2 * p]), __uint_as_float(v[2 * p + 1])));
              const float2 go = Codec<__nv_bfloat16>::unpack_word(gw);
              const float2 x = Codec<__nv_bfloat16>::unpack_word(hw[half * 8 + p]);
              w0[p] = Codec<__nv_bfloat16>::pack_word(bwd_math<float2, false, kF>(x, go, bc, acc_g));
            }
          }
          if (half == 0) {
            // the staging tile's previous TMA store has finished reading it
            if (lane == 0) bulk_wait_read<0>();
            __syncwarp();
          }
          if (kMode != kFwd || args.store_h) {
#pragma unroll
            for (int j = 0; j < 2; ++j)
              *reinterpret_cast<uint4*>(stage_out + sw64_offset(row, half * 2 + j)) =
                  make_uint4(w0[j * 4], w0[j * 4 + 1], w0[j * 4 + 2], w0[j * 4 + 3]);
          }
          if constexpr (kMode == kFwd) {
#pragma unroll
            for (int j = 0; j < 2; ++j)
              *reinterpret_cast<uint4*>(stage_out + kTileBytes + sw64_offset(row, half * 2 + j)) =
                  make_uint4(w1[j * 4], w1[j * 4 + 1], w1[j * 4 + 2], w1[j * 4 + 3]);
          }
        };
        // The second half's TMEM load is in flight while the first half is computed.
        const uint32_t col = uint32_t(acc * kBN + slice * kSlice + c * kChunk);
        uint32_t va[16];
        uint32_t vb[16];
        tmem_ld16(lane_addr + col, va);
        tmem_wait(va);
        tmem_ld16(lane_addr + col + kHalf, vb);
        do_half(va, 0);
        tmem_wait(vb);
        if (c == kChunksPerSlice - 1) {
          // this warp has read its part of the accumulator: hand it back to the MMA issuer
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if constexpr (kPair == 1) mbar_arrive(tempty + acc);
            else mbar_arrive_cluster(tempty0 + uint32_t(acc) * 8u);
          }
        }
        do_half(vb, 1);
        fence_async_shared();
        __syncwarp();
        if (lane == 0 && m0 < args.m) {  // rows past M: nothing to store (tail tile)
          if (kMode != kFwd || args.store_h) tma_store_2d(&tm_out0, stage_out, n0, m0);
          if constexpr (kMode == kFwd) tma_store_2d(&tm_out1, stage_out + kTileBytes, n0, m0);
          bulk_commit();
        }
      }
    }
    if constexpr (kMode == kBwd) {
      if (alive && cur_group >= 0) flush(cur_group);
    }
    if (lane == 0) bulk_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  if constexpr (kPair == 2) cluster_sync();  // the pair is done with TMEM and remote barriers
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_free<kPair>(tmem_base, kTmemCols);
  }
  if constexpr (kMode == kBwd) {
    // This CTA's warp rows, added in warp order into its row 0 (the reduction kernel then
    // reads one row per CTA).  The partial rows were written before the barrier above.
    if (threadIdx.x >= kEpiWarp0 * 32) {
      double* base = args.partial + size_t(blockIdx.x) * kEpiWarps * size_t(args.groups) * kAcc;
      const int n = args.groups * kAcc;
      for (int i = threadIdx.x - kEpiWarp0 * 32; i < n; i += kEpiWarps * 32) {
        double t = 0.0;
        for (int w = 0; w < kEpiWarps; ++w) t += base[size_t(w) * n + i];
        base[i] = t;
      }
    }
  }
}

// Coefficient gradients: one warp per group adds the CTA rows (row 0 of each CTA's block of
// row_stride warp rows) in a fixed order (lane-strided, then a fixed shuffle tree) and writes
// d_num / d_den with the sign conventions of the activation kernels.
constexpr int kReduceWarps = 8;
__global__ void __launch_bounds__(kReduceWarps * 32)
kat_gemm_reduce_kernel(const double* __restrict__ partial, int rows, int row_stride,
                       int groups, const float* __restrict__ den, float* __restrict__ d_num,
                       float* __restrict__ d_den, int formula) {
  const int g = blockIdx.x * kReduceWarps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (g >= groups) return;
  double tot[kAcc];
#pragma unroll
  for (int k = 0; k < kAcc; ++k) tot[k] = 0.0;
  for (int r = lane; r < rows; r += 32) {
    const double* src = partial + (size_t(r) * row_stride * groups + g) * kAcc;
#pragma unroll
    for (int k = 0; k < kAcc; ++k) tot[k] += src[k];
  }
#pragma unroll
  for (int k = 0; k < kAcc; ++k) {
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) tot[k] += __shfl_xor_sync(0xffffffffu, tot[k], m);
  }
  double v = 0.0;
#pragma unroll
  for (int k = 0; k < kAcc; ++k)
    if (lane == k) v = tot[k];
  if (lane >= kAcc) return;
  const float f = float(v);
  if (lane < 6) {
    d_num[g * 6 + lane] = f;
  } else {
    float sg = 1.0f;
    if (formula == kFormulaKat) {
      const float b = den[g * 4 + (lane - 6)];
      sg = b > 0.0f ? 1.0f : (b < 0.0f ? -1.0f : b * 0.0f);
    }
    d_den[g * 4 + (lane - 6)] = -(sg * f);
  }
}

// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encoder() {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// Row-major bf16 [rows, cols] matrix, box of box_rows x box_cols elements.
bool make_map(CUtensorMap* map, const void* ptr, int64_t rows, int64_t cols, uint32_t box_cols,
              uint32_t box_rows, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encoder();
  if (fn == nullptr) return false;
  const cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  const cuuint64_t strides[1] = {cuuint64_t(cols) * 2};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int sm_count(int device) {
  static std::mutex mu;
  static int cache[64] = {0};
  std::lock_guard<std::mutex> lock(mu);
  if (device < 0 || device >= 64) return 0;
  if (cache[device] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) != cudaSuccess)
      return 0;
    cache[device] = v;
  }
  return cache[device];
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_shape(int64_t m, int64_t n, int64_t k) {
  if (m < 0 || n < kBN || k < kBK) return KAT_ERR_BAD_SHAPE;
  if (n % kBN != 0 || k % kBK != 0) return KAT_ERR_BAD_SHAPE;
  if (m >= (int64_t(1) << 31) || n >= (int64_t(1) << 31) || k >= (int64_t(1) << 31))
    return KAT_ERR_BAD_SHAPE;
  const int64_t tiles = ((m + kBM - 1) / kBM) * (n / kBN);
  if (tiles >= (int64_t(1) << 31)) return KAT_ERR_BAD_SHAPE;
  return KAT_OK;
}

int check_groups(int64_t n, int32_t groups) {
  if (groups < 1 || n % groups != 0 || (n / groups) % kChunk != 0) return KAT_ERR_BAD_GROUPS;
  return KAT_OK;
}

// KAT_GEMM_CTA_PAIR=0 keeps one CTA per 128-row tile; by default a cluster's CTA pair shares
// each 256-row tile (cta_group::2) whenever the device can co-schedule CTA pairs.
bool pairs_enabled() {
  static const bool on = [] {
    const char* e = getenv("KAT_GEMM_CTA_PAIR");
    return !(e != nullptr && e[0] == '0');
  }();
  return on;
}

// Resident CTA pairs for this kernel on `device` (cluster occupancy, cached), or -1.
template <int kMode, int kF>
int pair_slots(int device) {
  static std::mutex mu;
  static int cache[64] = {0};
  if (device < 0 || device >= 64) return -1;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[device] == 0) {
    auto kernel = kat_gemm_kernel<kMode, kF, 2>;
    constexpr uint32_t smem = smem_bytes<kMode, 2>();
    int clusters = -1;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) ==
        cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      cfg.blockDim = dim3(threads_of<kMode>());
      cfg.dynamicSmemBytes = smem;
      cfg.gridDim = dim3(2 * uint32_t(sm_count(device) / 2));
      int c = 0;
      if (cudaOccupancyMaxActiveClusters(&c, kernel, &cfg) == cudaSuccess && c > 0) clusters = c;
    }
    cudaGetLastError();
    cache[device] = clusters;
  }
  return cache[device];
}

// Test hook, off unless kat_gemm_set_test_stall turned it on in this process: the next
// launches' MMA issuer waits on a barrier nothing completes (the bounded-wait path).
std::atomic<int> g_test_stall{0};

template <int kMode, int kF, int kPair>
int launch_mode(const CUtensorMap& ma, const void* b, int64_t m, int64_t n, int64_t k,
                const CUtensorMap& o0, const CUtensorMap& o1, const CUtensorMap& h,
                GemmArgs args, int device, cudaStream_t stream, int* grid_out) {
  auto kernel = kat_gemm_kernel<kMode, kF, kPair>;
  constexpr uint32_t smem = smem_bytes<kMode, kPair>();
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) !=
      cudaSuccess)
    return KAT_ERR_CUDA;
  CUtensorMap mb;
  if (!make_map(&mb, b, n, k, kBK, uint32_t(kBN / kPair), CU_TENSOR_MAP_SWIZZLE_128B))
    return KAT_ERR_CUDA;
  args.stall = g_test_stall.load(std::memory_order_relaxed);
  args.m_tiles = int32_t((m + kBM * kPair - 1) / (kBM * kPair));
  args.num_tiles = int32_t(int64_t(args.m_tiles) * (n / kBN));
  const int sms = sm_count(device);
  if (sms <= 0) return KAT_ERR_CUDA;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.blockDim = dim3(threads_of<kMode>());
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  int slots = sms;
  if constexpr (kPair == 2) {
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    slots = pair_slots<kMode, kF>(device);
    if (slots < 1) return KAT_ERR_CUDA;
  }
  if (slots > args.num_tiles) slots = args.num_tiles;
  cfg.gridDim = dim3(uint32_t(slots * kPair));
  if (cudaLaunchKernelEx(&cfg, kernel, ma, mb, o0, o1, h, args) != cudaSuccess)
    return KAT_ERR_CUDA;
  *grid_out = slots * kPair;
  return cudaGetLastError() == cudaSuccess ? KAT_OK : KAT_ERR_CUDA;
}

// One CTA pair per 256-row tile when that takes no more waves of tiles than one CTA per
// 128-row tile (pairs halve each CTA's B traffic, but a ragged last wave costs a whole tile
// time), else one CTA per tile.  Every mode decides the same way for the same M, N, so the
// plain GEMM and the fused kernels share their accumulation order.
template <int kMode, int kF>
int launch(const CUtensorMap& ma, const void* b, int64_t m, int64_t n, int64_t k,
           const CUtensorMap& o0, const CUtensorMap& o1, const CUtensorMap& h,
           const GemmArgs& args, int device, cudaStream_t stream, int* grid_out) {
  if (pairs_enabled()) {
    const int pairs = pair_slots<kPlain, kFormulaKat>(device);
    const int sms = sm_count(device);
    if (pairs > 0 && sms > 0) {
      const int64_t t1 = ((m + kBM - 1) / kBM) * (n / kBN);
      const int64_t t2 = ((m + 2 * kBM - 1) / (2 * kBM)) * (n / kBN);
      const int64_t waves1 = (t1 + sms - 1) / sms;
      const int64_t waves2 = (t2 + pairs - 1) / pairs;
      if (waves2 <= waves1) {
        const int rc = launch_mode<kMode, kF, 2>(ma, b, m, n, k, o0, o1, h, args, device,
                                                stream, grid_out);
        if (rc == KAT_OK) return rc;
        cudaGetLastError();  // clear a refused cluster launch before the single-CTA launch
      }
    }
  }
  return launch_mode<kMode, kF, 1>(ma, b, m, n, k, o0, o1, h, args, device, stream, grid_out);
}

int current_device(int* dev) { return cudaGetDevice(dev) == cudaSuccess ? KAT_OK : KAT_ERR_CUDA; }

}  // namespace

// ---------------------------------------------------------------------------
// C ABI.
// ---------------------------------------------------------------------------

extern "C" {

int kat_gemm_bf16(const void* a, const void* b, const void* bias, void* c, int64_t m, int64_t n,
                  int64_t k, void* stream) {
  if (a == nullptr || b == nullptr || c == nullptr) return KAT_ERR_NULL_POINTER;
  if (int st = check_shape(m, n, k)) return st;
  if (!aligned16(a) || !aligned16(b) || !aligned16(c) || (bias != nullptr && !aligned16(bias)))
    return KAT_ERR_BAD_SHAPE;
  if (m == 0) return KAT_OK;  // empty problem: nothing to do
  int dev = 0;
  if (int st = current_device(&dev)) return st;
  CUtensorMap ma, mc;
  if (!make_map(&ma, a, m, k, kBK, kBM, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map(&mc, c, m, n, kChunk, kWarpRows, CU_TENSOR_MAP_SWIZZLE_64B))
    return KAT_ERR_CUDA;
  GemmArgs args{};
  args.m = int32_t(m);
  args.n_tiles = int32_t(n / kBN);
  args.k_blocks = int32_t(k / kBK);
  args.group_width = int32_t(n);
  args.groups = 1;
  args.bias = static_cast<const uint16_t*>(bias);
  int grid = 0;
  return launch<kPlain, kFormulaKat>(ma, b, m, n, k, mc, mc, mc, args, dev,
                                     static_cast<cudaStream_t>(stream), &grid);
}

int kat_gemm_rational_fwd(const void* a, const void* b, const void* bias, const float* num,
                          const float* den, void* h, void* y, int64_t m, int64_t n, int64_t k,
                          int32_t num_groups, int32_t formula, void* stream) {
  if (a == nullptr || b == nullptr || num == nullptr || den == nullptr || y == nullptr)
    return KAT_ERR_NULL_POINTER;
  if (formula != KAT_FORMULA_KAT && formula != KAT_FORMULA_ABS_SUM) return KAT_ERR_BAD_FORMULA;
  if (int st = check_shape(m, n, k)) return st;
  if (int st = check_groups(n, num_groups)) return st;
  if (!aligned16(a) || !aligned16(b) || (h != nullptr && !aligned16(h)) || !aligned16(y) ||
      (bias != nullptr && !aligned16(bias)))
    return KAT_ERR_BAD_SHAPE;
  if (m == 0) return KAT_OK;  // empty problem: nothing to do
  int dev = 0;
  if (int st = current_device(&dev)) return st;
  CUtensorMap ma, mh, my;
  if (!make_map(&ma, a, m, k, kBK, kBM, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map(&mh, h != nullptr ? h : y, m, n, kChunk, kWarpRows, CU_TENSOR_MAP_SWIZZLE_64B) ||
      !make_map(&my, y, m, n, kChunk, kWarpRows, CU_TENSOR_MAP_SWIZZLE_64B))
    return KAT_ERR_CUDA;
  GemmArgs args{};
  args.m = int32_t(m);
  args.store_h = h != nullptr ? 1 : 0;
  args.n_tiles = int32_t(n / kBN);
  args.k_blocks = int32_t(k / kBK);
  args.group_width = int32_t(n / num_groups);
  args.groups = num_groups;
  args.bias = static_cast<const uint16_t*>(bias);
  args.num = num;
  args.den = den;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int grid = 0;
  return formula == KAT_FORMULA_KAT
             ? launch<kFwd, kFormulaKat>(ma, b, m, n, k, mh, my, mh, args, dev, st, &grid)
             : launch<kFwd, kFormulaAbsSum>(ma, b, m, n, k, mh, my, mh, args, dev, st, &grid);
}

size_t kat_gemm_rational_bwd_workspace_bytes(int64_t m, int64_t n, int32_t num_groups,
                                             int device) {
  if (check_shape(m, n, kBK) != KAT_OK || num_groups < 1) return 0;
  const int sms = sm_count(device);  // the grid never exceeds one CTA per SM
  if (sms <= 0) return 0;
  return size_t(sms) * kMaxEpiWarps * size_t(num_groups) * kAcc * sizeof(double);
}

int kat_gemm_rational_bwd(const void* a, const void* b, const void* h, const float* num,
                          const float* den, void* dh, float* d_num, float* d_den,
                          void* workspace, size_t workspace_bytes, int64_t m, int64_t n,
                          int64_t k, int32_t num_groups, int32_t formula, void* stream) {
  if (a == nullptr || b == nullptr || h == nullptr || num == nullptr || den == nullptr ||
      dh == nullptr || d_num == nullptr || d_den == nullptr)
    return KAT_ERR_NULL_POINTER;
  if (formula != KAT_FORMULA_KAT && formula != KAT_FORMULA_ABS_SUM) return KAT_ERR_BAD_FORMULA;
  if (int st = check_shape(m, n, k)) return st;
  if (int st = check_groups(n, num_groups)) return st;
  if (!aligned16(a) || !aligned16(b) || !aligned16(h) || !aligned16(dh)) return KAT_ERR_BAD_SHAPE;
  if (m == 0) {  // empty problem: the coefficient gradients are zero sums
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (cudaMemsetAsync(d_num, 0, size_t(num_groups) * 6 * sizeof(float), st) != cudaSuccess ||
        cudaMemsetAsync(d_den, 0, size_t(num_groups) * 4 * sizeof(float), st) != cudaSuccess)
      return KAT_ERR_CUDA;
    return KAT_OK;
  }
  int dev = 0;
  if (int st = current_device(&dev)) return st;
  const int sms = sm_count(dev);
  if (sms <= 0) return KAT_ERR_CUDA;
  const size_t need = size_t(sms) * kMaxEpiWarps * size_t(num_groups) * kAcc * sizeof(double);
  if (workspace == nullptr || workspace_bytes < need || !aligned16(workspace))
    return KAT_ERR_WORKSPACE;
  CUtensorMap ma, mh, md;
  if (!make_map(&ma, a, m, k, kBK, kBM, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map(&mh, h, m, n, kChunk, kWarpRows, CU_TENSOR_MAP_SWIZZLE_64B) ||
      !make_map(&md, dh, m, n, kChunk, kWarpRows, CU_TENSOR_MAP_SWIZZLE_64B))
    return KAT_ERR_CUDA;
  GemmArgs args{};
  args.m = int32_t(m);
  args.n_tiles = int32_t(n / kBN);
  args.k_blocks = int32_t(k / kBK);
  args.group_width = int32_t(n / num_groups);
  args.groups = num_groups;
  args.num = num;
  args.den = den;
  args.partial = static_cast<double*>(workspace);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int grid = 0;
  const int rc = formula == KAT_FORMULA_KAT
                     ? launch<kBwd, kFormulaKat>(ma, b, m, n, k, md, md, mh, args, dev, st, &grid)
                     : launch<kBwd, kFormulaAbsSum>(ma, b, m, n, k, md, md, mh, args, dev, st,
                                                    &grid);
  if (rc != KAT_OK) return rc;
  const int rgrid = (num_groups + kReduceWarps - 1) / kReduceWarps;
  kat_gemm_reduce_kernel<<<rgrid, kReduceWarps * 32, 0, st>>>(
      static_cast<const double*>(workspace), grid, Cfg<kBwd>::kEpiWarps, num_groups, den, d_num, d_den, formula);
  return cudaGetLastError() == cudaSuccess ? KAT_OK : KAT_ERR_CUDA;
}

int kat_gemm_set_test_stall(int on) {
  g_test_stall.store(on ? 1 : 0, std::memory_order_relaxed);
  return KAT_OK;
}

int kat_gemm_device_status(int device, int reset, int* status) {
  if (status == nullptr) return KAT_ERR_NULL_POINTER;
  int prev = 0;
  if (cudaGetDevice(&prev) != cudaSuccess) return KAT_ERR_CUDA;
  if (device != prev && cudaSetDevice(device) != cudaSuccess) return KAT_ERR_CUDA;
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_gemm_status, sizeof(int));
  if (e == cudaSuccess && reset) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_gemm_status, &zero, sizeof(int));
  }
  if (device != prev) cudaSetDevice(prev);
  if (e != cudaSuccess) return KAT_ERR_CUDA;
  *status = v;
  return KAT_OK;
}

}  // extern "C"
