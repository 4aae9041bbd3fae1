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
#include <string.h>

#include <map>
#include <type_traits>
#include <mutex>
#include <tuple>

#include "kat_rational.h"

namespace {

constexpr int kAcc = 10;          // 6 numerator + 4 denominator gradient sums
constexpr int kMaxThreads = 512;  // block size cap
constexpr int kReduceThreads = kAcc * 32;
constexpr int64_t kMaxElements = int64_t(1) << 48;
constexpr int64_t kMaxBlocks = int64_t(1) << 14;

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
};

// ---------------------------------------------------------------------------
// Element I/O: a vector of V elements <-> float[V].
// ---------------------------------------------------------------------------

template <int BYTES> struct BitsOf;
template <> struct BitsOf<16> { using T = uint4; };
template <> struct BitsOf<8> { using T = uint2; };
template <> struct BitsOf<4> { using T = uint32_t; };
template <> struct BitsOf<2> { using T = uint16_t; };

template <typename B> __device__ __forceinline__ void bits_to_words(const B& b, uint32_t* w);
template <> __device__ __forceinline__ void bits_to_words<uint4>(const uint4& b, uint32_t* w) {
  w[0] = b.x; w[1] = b.y; w[2] = b.z; w[3] = b.w;
}
template <> __device__ __forceinline__ void bits_to_words<uint2>(const uint2& b, uint32_t* w) {
  w[0] = b.x; w[1] = b.y;
}
template <> __device__ __forceinline__ void bits_to_words<uint32_t>(const uint32_t& b, uint32_t* w) {
  w[0] = b;
}
template <typename B> __device__ __forceinline__ B words_to_bits(const uint32_t* w);
template <> __device__ __forceinline__ uint4 words_to_bits<uint4>(const uint32_t* w) {
  return make_uint4(w[0], w[1], w[2], w[3]);
}
template <> __device__ __forceinline__ uint2 words_to_bits<uint2>(const uint32_t* w) {
  return make_uint2(w[0], w[1]);
}
template <> __device__ __forceinline__ uint32_t words_to_bits<uint32_t>(const uint32_t* w) {
  return w[0];
}

template <typename Tio> struct Codec;

template <> struct Codec<float> {
  static constexpr int kBytes = 4;
  __device__ __forceinline__ static float2 unpack2(uint32_t lo, uint32_t hi) {
    return make_float2(__uint_as_float(lo), __uint_as_float(hi));
  }
  __device__ __forceinline__ static float unpack1(uint32_t v) { return __uint_as_float(v); }
  __device__ __forceinline__ static uint32_t pack1(float f) { return __float_as_uint(f); }
};

template <> struct Codec<__nv_bfloat16> {
  static constexpr int kBytes = 2;
  __device__ __forceinline__ static float2 unpack_word(uint32_t w) {
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
  }
  __device__ __forceinline__ static uint32_t pack_word(float2 f) {
    __nv_bfloat162 h = __floats2bfloat162_rn(f.x, f.y);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ __forceinline__ static float unpack1(uint16_t v) {
    return __uint_as_float(uint32_t(v) << 16);
  }
  __device__ __forceinline__ static uint16_t pack1(float f) {
    __nv_bfloat16 h = __float2bfloat16_rn(f);
    return *reinterpret_cast<uint16_t*>(&h);
  }
};

template <> struct Codec<__half> {
  static constexpr int kBytes = 2;
  __device__ __forceinline__ static float2 unpack_word(uint32_t w) {
    __half2 h = *reinterpret_cast<__half2*>(&w);
    return __half22float2(h);
  }
  __device__ __forceinline__ static uint32_t pack_word(float2 f) {
    __half2 h = __floats2half2_rn(f.x, f.y);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ __forceinline__ static float unpack1(uint16_t v) {
    __half h = *reinterpret_cast<__half*>(&v);
    return __half2float(h);
  }
  __device__ __forceinline__ static uint16_t pack1(float f) {
    __half h = __float2half_rn(f);
    return *reinterpret_cast<uint16_t*>(&h);
  }
};

// A vector of V elements held as V/2 float2 pairs (V even) or one float (V == 1).
template <int V> struct Frag {
  static constexpr int kPairs = V / 2;
  float2 p[kPairs];
};
template <> struct Frag<1> {
  float s;
};

// Raw bits of one vector: what a single load / store moves.
template <typename Tio, int V> struct RawOf {
  using T = typename BitsOf<V * sizeof(Tio)>::T;
};
template <> struct RawOf<float, 1> { using T = uint32_t; };

template <typename Tio, int V>
__device__ __forceinline__ typename RawOf<Tio, V>::T load_raw(const Tio* __restrict__ ptr) {
  using B = typename RawOf<Tio, V>::T;
  if constexpr (sizeof(B) == 2) {
    return __ldg(reinterpret_cast<const unsigned short*>(ptr));
  } else {
    return __ldg(reinterpret_cast<const B*>(ptr));
  }
}

template <typename Tio, int V>
__device__ __forceinline__ void store_raw(Tio* __restrict__ ptr, typename RawOf<Tio, V>::T b) {
  using B = typename RawOf<Tio, V>::T;
  *reinterpret_cast<B*>(ptr) = b;
}

template <typename Tio, int V>
__device__ __forceinline__ Frag<V> unpack(typename RawOf<Tio, V>::T b) {
  Frag<V> f;
  if constexpr (V == 1) {
    if constexpr (sizeof(Tio) == 4) {
      f.s = __uint_as_float(b);
    } else {
      f.s = Codec<Tio>::unpack1(b);
    }
  } else if constexpr (sizeof(Tio) == 4) {
    uint32_t w[V];
    bits_to_words(b, w);
#pragma unroll
    for (int i = 0; i < V / 2; ++i) f.p[i] = Codec<float>::unpack2(w[2 * i], w[2 * i + 1]);
  } else {
    uint32_t w[V / 2];
    bits_to_words(b, w);
#pragma unroll
    for (int i = 0; i < V / 2; ++i) f.p[i] = Codec<Tio>::unpack_word(w[i]);
  }
  return f;
}

template <typename Tio, int V>
__device__ __forceinline__ typename RawOf<Tio, V>::T pack(const Frag<V>& f) {
  using B = typename RawOf<Tio, V>::T;
  if constexpr (V == 1) {
    if constexpr (sizeof(Tio) == 4) {
      return __float_as_uint(f.s);
    } else {
      return Codec<Tio>::pack1(f.s);
    }
  } else if constexpr (sizeof(Tio) == 4) {
    uint32_t w[V];
#pragma unroll
    for (int i = 0; i < V / 2; ++i) {
      w[2 * i] = __float_as_uint(f.p[i].x);
      w[2 * i + 1] = __float_as_uint(f.p[i].y);
    }
    return words_to_bits<B>(w);
  } else {
    uint32_t w[V / 2];
#pragma unroll
    for (int i = 0; i < V / 2; ++i) w[i] = Codec<Tio>::pack_word(f.p[i]);
    return words_to_bits<B>(w);
  }
}

// ---------------------------------------------------------------------------
// Scalar / paired arithmetic.
// ---------------------------------------------------------------------------

__device__ __forceinline__ float fma_(float a, float b, float c) { return __fmaf_rn(a, b, c); }
__device__ __forceinline__ float2 fma_(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float mul_(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float2 mul_(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float add_(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float2 add_(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float neg_(float a) { return -a; }
__device__ __forceinline__ float2 neg_(float2 a) { return make_float2(-a.x, -a.y); }

// PTX rcp.approx.ftz.f32: reciprocal with at most 1 ulp error (subnormal
// inputs flush to zero, giving +-inf).
__device__ __forceinline__ float rcp_(float q) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(q));
  return r;
}
__device__ __forceinline__ float2 rcp_(float2 q) { return make_float2(rcp_(q.x), rcp_(q.y)); }
__device__ __forceinline__ float div_rn_(float a, float b) { return __fdiv_rn(a, b); }
__device__ __forceinline__ float2 div_rn_(float2 a, float2 b) {
  return make_float2(__fdiv_rn(a.x, b.x), __fdiv_rn(a.y, b.y));
}

template <typename L> __device__ __forceinline__ L bcast(float v);
template <> __device__ __forceinline__ float bcast<float>(float v) { return v; }
template <> __device__ __forceinline__ float2 bcast<float2>(float v) { return make_float2(v, v); }

__device__ __forceinline__ float lane_sum(float v) { return v; }
__device__ __forceinline__ float lane_sum(float2 v) { return v.x + v.y; }

// Coefficients of one group, broadcast to the lane type.
template <typename L> struct FwdCoef {
  L a0, a1, a2, a3, a4, a5;  // numerator
  L c1, c2, c3, c4;          // |b_i|
  L one;
};

template <typename L> struct BwdCoef {
  L a0, a1, a2, a3, a4, a5;  // numerator
  L c1, c2, c3, c4;          // |b_i|
  L p1, p2, p3, p4, p5;      // k * a_k: coefficients of P'
  L q2, q3, q4;              // i * |b_i| for i = 2..4 (q1 = c1): coefficients of Q'
  L one;
};

template <typename L>
__device__ __forceinline__ void load_fwd_coef(const float* __restrict__ num,
                                              const float* __restrict__ den, int64_t g,
                                              FwdCoef<L>& c) {
  const float* a = num + g * 6;
  const float* b = den + g * 4;
  c.a0 = bcast<L>(__ldg(a + 0)); c.a1 = bcast<L>(__ldg(a + 1)); c.a2 = bcast<L>(__ldg(a + 2));
  c.a3 = bcast<L>(__ldg(a + 3)); c.a4 = bcast<L>(__ldg(a + 4)); c.a5 = bcast<L>(__ldg(a + 5));
  c.c1 = bcast<L>(fabsf(__ldg(b + 0))); c.c2 = bcast<L>(fabsf(__ldg(b + 1)));
  c.c3 = bcast<L>(fabsf(__ldg(b + 2))); c.c4 = bcast<L>(fabsf(__ldg(b + 3)));
  c.one = bcast<L>(1.0f);
}

template <typename L>
__device__ __forceinline__ void load_bwd_coef(const float* __restrict__ num,
                                              const float* __restrict__ den, int64_t g,
                                              BwdCoef<L>& c) {
  const float* a = num + g * 6;
  const float* b = den + g * 4;
  const float a0 = __ldg(a + 0), a1 = __ldg(a + 1), a2 = __ldg(a + 2);
  const float a3 = __ldg(a + 3), a4 = __ldg(a + 4), a5 = __ldg(a + 5);
  const float c1 = fabsf(__ldg(b + 0)), c2 = fabsf(__ldg(b + 1));
  const float c3 = fabsf(__ldg(b + 2)), c4 = fabsf(__ldg(b + 3));
  c.a0 = bcast<L>(a0); c.a1 = bcast<L>(a1); c.a2 = bcast<L>(a2);
  c.a3 = bcast<L>(a3); c.a4 = bcast<L>(a4); c.a5 = bcast<L>(a5);
  c.c1 = bcast<L>(c1); c.c2 = bcast<L>(c2); c.c3 = bcast<L>(c3); c.c4 = bcast<L>(c4);
  c.p1 = bcast<L>(a1); c.p2 = bcast<L>(2.0f * a2); c.p3 = bcast<L>(3.0f * a3);
  c.p4 = bcast<L>(4.0f * a4); c.p5 = bcast<L>(5.0f * a5);
  c.q2 = bcast<L>(2.0f * c2); c.q3 = bcast<L>(3.0f * c3); c.q4 = bcast<L>(4.0f * c4);
  c.one = bcast<L>(1.0f);
}

// Forward on one lane (scalar or pair).
template <typename L, bool kExactDiv>
__device__ __forceinline__ L fwd_math(L x, const FwdCoef<L>& c) {
  L p = fma_(c.a5, x, c.a4);
  p = fma_(p, x, c.a3);
  p = fma_(p, x, c.a2);
  p = fma_(p, x, c.a1);
  p = fma_(p, x, c.a0);
  L q = fma_(c.c4, x, c.c3);
  q = fma_(q, x, c.c2);
  q = fma_(q, x, c.c1);
  q = fma_(q, x, c.one);
  if constexpr (kExactDiv) {
    return div_rn_(p, q);
  } else {
    return mul_(p, rcp_(q));
  }
}

// Backward on one lane: returns dx and adds this lane's gradient terms into
// acc[0..5] (sum u x^k) and acc[6..9] (sum u y x^i, i = 1..4).
template <typename L, bool kRefine>
__device__ __forceinline__ L bwd_math(L x, L go, const BwdCoef<L>& c, L (&acc)[kAcc]) {
  L p = fma_(c.a5, x, c.a4);
  p = fma_(p, x, c.a3);
  p = fma_(p, x, c.a2);
  p = fma_(p, x, c.a1);
  p = fma_(p, x, c.a0);
  L q = fma_(c.c4, x, c.c3);
  q = fma_(q, x, c.c2);
  q = fma_(q, x, c.c1);
  q = fma_(q, x, c.one);
  L dp = fma_(c.p5, x, c.p4);
  dp = fma_(dp, x, c.p3);
  dp = fma_(dp, x, c.p2);
  dp = fma_(dp, x, c.p1);
  L dq = fma_(c.q4, x, c.q3);
  dq = fma_(dq, x, c.q2);
  dq = fma_(dq, x, c.c1);
  L r = rcp_(q);
  if constexpr (kRefine) {  // Newton-Raphson: r <- r + r (1 - q r)
    const L e = fma_(neg_(q), r, c.one);
    r = fma_(r, e, r);
  }
  const L u = mul_(go, r);         // go / Q
  const L y = mul_(p, r);          // P / Q
  const L t = fma_(neg_(y), dq, dp);  // P' - y Q'
  const L w = mul_(u, y);          // go P / Q^2
  const L x2 = mul_(x, x);
  const L x3 = mul_(x2, x);
  const L x4 = mul_(x2, x2);
  const L x5 = mul_(x4, x);
  acc[0] = add_(acc[0], u);
  acc[1] = fma_(u, x, acc[1]);
  acc[2] = fma_(u, x2, acc[2]);
  acc[3] = fma_(u, x3, acc[3]);
  acc[4] = fma_(u, x4, acc[4]);
  acc[5] = fma_(u, x5, acc[5]);
  acc[6] = fma_(w, x, acc[6]);
  acc[7] = fma_(w, x2, acc[7]);
  acc[8] = fma_(w, x3, acc[8]);
  acc[9] = fma_(w, x4, acc[9]);
  return mul_(u, t);
}

// One vector through the forward / backward math.
template <typename Tio, int V, typename L, bool kExact>
__device__ __forceinline__ typename RawOf<Tio, V>::T fwd_vec(typename RawOf<Tio, V>::T raw,
                                                             const FwdCoef<L>& c) {
  Frag<V> f = unpack<Tio, V>(raw);
  if constexpr (V == 1) {
    f.s = fwd_math<float, kExact>(f.s, c);
  } else {
#pragma unroll
    for (int k = 0; k < V / 2; ++k) f.p[k] = fwd_math<float2, kExact>(f.p[k], c);
  }
  return pack<Tio, V>(f);
}

template <typename Tio, int V, typename L, bool kRefine>
__device__ __forceinline__ typename RawOf<Tio, V>::T bwd_vec(typename RawOf<Tio, V>::T rx,
                                                             typename RawOf<Tio, V>::T rg,
                                                             const BwdCoef<L>& c,
                                                             L (&acc)[kAcc]) {
  Frag<V> fx = unpack<Tio, V>(rx);
  const Frag<V> fg = unpack<Tio, V>(rg);
  if constexpr (V == 1) {
    fx.s = bwd_math<float, kRefine>(fx.s, fg.s, c, acc);
  } else {
#pragma unroll
    for (int k = 0; k < V / 2; ++k) fx.p[k] = bwd_math<float2, kRefine>(fx.p[k], fg.p[k], c, acc);
  }
  return pack<Tio, V>(fx);
}

// Item range [i0, i1) of block `blk` (even split, sizes differ by at most one).
__device__ __forceinline__ void block_items(const Plan& p, int64_t blk, int64_t& i0, int64_t& i1) {
  i0 = p.items * blk / p.blocks;
  i1 = p.items * (blk + 1) / p.blocks;
}

// ---------------------------------------------------------------------------
// Forward kernel.
// ---------------------------------------------------------------------------

template <typename Tio, int V, int U>
__global__ void __launch_bounds__(kMaxThreads)
kat_fwd_kernel(const Tio* __restrict__ x, Tio* __restrict__ y,
               const float* __restrict__ num, const float* __restrict__ den, const Plan p) {
  using L = typename std::conditional<V == 1, float, float2>::type;
  using Raw = typename RawOf<Tio, V>::T;
  constexpr bool kExact = sizeof(Tio) == 4;
  const int tc = threadIdx.x % p.tile_cols;
  const int tr = threadIdx.x / p.tile_cols;
  if (tr >= p.tile_rows) return;
  int64_t i0, i1;
  block_items(p, blockIdx.x, i0, i1);
  const int64_t row_step = int64_t(p.tile_rows) * p.width;
  for (int64_t i = i0; i < i1;) {
    const int64_t cb = i / p.rows;
    const int64_t seg_end = min(i1, (cb + 1) * p.rows);
    const int64_t col = cb * p.tile_cols + tc;
    if (col < p.vec_cols) {
      FwdCoef<L> c;
      load_fwd_coef<L>(num, den, col / p.vec_group, c);
      const int64_t r1 = seg_end - cb * p.rows;
      int64_t r = i - cb * p.rows + tr;
      const int64_t off = r * p.width + col * V;
      const Tio* xp = x + off;
      Tio* yp = y + off;
#pragma unroll 1
      for (; r + (U - 1) * p.tile_rows < r1; r += U * p.tile_rows) {
        Raw raw[U];
#pragma unroll
        for (int u = 0; u < U; ++u) raw[u] = load_raw<Tio, V>(xp + u * row_step);
#pragma unroll
        for (int u = 0; u < U; ++u) {
          store_raw<Tio, V>(yp + u * row_step, fwd_vec<Tio, V, L, kExact>(raw[u], c));
        }
        xp += U * row_step;
        yp += U * row_step;
      }
#pragma unroll 1
      for (; r < r1; r += p.tile_rows) {
        store_raw<Tio, V>(yp, fwd_vec<Tio, V, L, kExact>(load_raw<Tio, V>(xp), c));
        xp += row_step;
        yp += row_step;
      }
    }
    i = seg_end;
  }
}

// ---------------------------------------------------------------------------
// Backward kernel (dx + per-block partial coefficient sums).
// ---------------------------------------------------------------------------

template <typename Tio, int V, int U>
__global__ void __launch_bounds__(kMaxThreads)
kat_bwd_kernel(const Tio* __restrict__ x, const Tio* __restrict__ gy, Tio* __restrict__ dx,
               const float* __restrict__ num, const float* __restrict__ den,
               double* __restrict__ partial, const Plan p) {
  using L = typename std::conditional<V == 1, float, float2>::type;
  using Raw = typename RawOf<Tio, V>::T;
  constexpr bool kRefine = sizeof(Tio) == 4;
  __shared__ float s_acc[kAcc][kMaxThreads];

  const int tc = threadIdx.x % p.tile_cols;
  const int tr = threadIdx.x / p.tile_cols;
  const bool row_thread = tr < p.tile_rows;
  const bool write_dx = dx != nullptr;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;

  int64_t i0, i1;
  block_items(p, blockIdx.x, i0, i1);
  const int64_t row_step = int64_t(p.tile_rows) * p.width;
  const int64_t cb0 = i0 / p.rows;

  for (int64_t i = i0; i < i1;) {
    const int64_t cb = i / p.rows;
    const int64_t seg_end = min(i1, (cb + 1) * p.rows);
    const int64_t col = cb * p.tile_cols + tc;
    L acc[kAcc];
#pragma unroll
    for (int k = 0; k < kAcc; ++k) acc[k] = bcast<L>(0.0f);

    if (row_thread && col < p.vec_cols) {
      BwdCoef<L> c;
      load_bwd_coef<L>(num, den, col / p.vec_group, c);
      const int64_t r1 = seg_end - cb * p.rows;
      int64_t r = i - cb * p.rows + tr;
      const int64_t off = r * p.width + col * V;
      const Tio* xp = x + off;
      const Tio* gp = gy + off;
      Tio* dp = write_dx ? dx + off : nullptr;
#pragma unroll 1
      for (; r + (U - 1) * p.tile_rows < r1; r += U * p.tile_rows) {
        Raw rx[U], rg[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          rx[u] = load_raw<Tio, V>(xp + u * row_step);
          rg[u] = load_raw<Tio, V>(gp + u * row_step);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const Raw d = bwd_vec<Tio, V, L, kRefine>(rx[u], rg[u], c, acc);
          if (write_dx) store_raw<Tio, V>(dp + u * row_step, d);
        }
        xp += U * row_step;
        gp += U * row_step;
        if (write_dx) dp += U * row_step;
      }
#pragma unroll 1
      for (; r < r1; r += p.tile_rows) {
        const Raw d = bwd_vec<Tio, V, L, kRefine>(load_raw<Tio, V>(xp), load_raw<Tio, V>(gp), c, acc);
        if (write_dx) store_raw<Tio, V>(dp, d);
        xp += row_step;
        gp += row_step;
        if (write_dx) dp += row_step;
      }
    }

    // Block reduction of this segment, per group, in a fixed order.
#pragma unroll
    for (int k = 0; k < kAcc; ++k) s_acc[k][threadIdx.x] = lane_sum(acc[k]);
    __syncthreads();
    const int64_t col0 = cb * p.tile_cols;
    const int64_t col_end = min(col0 + p.tile_cols, p.vec_cols);
    const int64_t g_first = col0 / p.vec_group;
    const int64_t g_last = (col_end - 1) / p.vec_group;
    const int n_out = int(g_last - g_first + 1) * kAcc;
    const int64_t seg = cb - cb0;
    for (int o = warp; o < n_out; o += nwarps) {
      const int lg = o / kAcc;
      const int k = o - lg * kAcc;
      const int64_t g = g_first + lg;
      const int tlo = int(max(g * p.vec_group, col0) - col0);
      const int thi = int(min((g + 1) * p.vec_group, col_end) - col0);
      const int wcols = thi - tlo;
      const int n = wcols * p.tile_rows;
      double s = 0.0;
      for (int j = lane; j < n; j += 32) {
        const int jr = j / wcols;
        const int jc = tlo + (j - jr * wcols);
        s += double(s_acc[k][jr * p.tile_cols + jc]);
      }
#pragma unroll
      for (int m = 16; m > 0; m >>= 1) s += __shfl_xor_sync(0xffffffffu, s, m);
      if (lane == 0) {
        partial[((int64_t(blockIdx.x) * p.max_segments + seg) * p.max_local_groups + lg) * kAcc + k] = s;
      }
    }
    __syncthreads();
    i = seg_end;
  }
}

// Grid reduction: one block per group, warp k sums coefficient slot k over all
// blocks in block order (lane j takes blocks j, j+32, ...; fixed xor tree).
__global__ void __launch_bounds__(kReduceThreads)
kat_bwd_reduce_kernel(const double* __restrict__ partial, const float* __restrict__ den,
                      float* __restrict__ dnum, float* __restrict__ dden, const Plan p) {
  const int64_t g = blockIdx.x;
  const int k = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  double s = 0.0;
  for (int64_t blk = lane; blk < p.blocks; blk += 32) {
    int64_t i0, i1;
    block_items(p, blk, i0, i1);
    const int64_t cb0 = i0 / p.rows;
    const int64_t cb1 = (i1 - 1) / p.rows;
    for (int64_t cb = cb0; cb <= cb1; ++cb) {
      const int64_t col0 = cb * p.tile_cols;
      const int64_t col_end = min(col0 + p.tile_cols, p.vec_cols);
      const int64_t g_first = col0 / p.vec_group;
      const int64_t g_last = (col_end - 1) / p.vec_group;
      if (g < g_first) break;
      if (g > g_last) continue;
      s += partial[((blk * p.max_segments + (cb - cb0)) * p.max_local_groups + (g - g_first)) * kAcc + k];
    }
  }
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) s += __shfl_xor_sync(0xffffffffu, s, m);
  if (lane == 0) {
    const float v = float(s);
    if (k < 6) {
      dnum[g * 6 + k] = v;
    } else {
      const float b = den[g * 4 + (k - 6)];
      // sgn(b) with sgn(0) = 0 and sgn(NaN) = NaN, as torch.sgn.
      const float sg = b > 0.0f ? 1.0f : (b < 0.0f ? -1.0f : b * 0.0f);
      dden[g * 4 + (k - 6)] = -(sg * v);
    }
  }
}

// ---------------------------------------------------------------------------
// Host side: validation, planning, dispatch.
// ---------------------------------------------------------------------------

constexpr int kUnroll = 4;

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
                   int vec, int sm_count, int ctas_per_sm, Plan* p) {
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
  if (p->vec_cols <= kMaxThreads) {
    p->tile_cols = int32_t(p->vec_cols);
    int64_t tr = kMaxThreads / p->tile_cols;
    if (tr > batch) tr = batch;
    if (tr < 1) tr = 1;
    p->tile_rows = int32_t(tr);
  } else {
    const int64_t ncb = (p->vec_cols + kMaxThreads - 1) / kMaxThreads;
    int64_t tcols = (p->vec_cols + ncb - 1) / ncb;
    tcols = (tcols + 31) / 32 * 32;
    if (tcols > kMaxThreads) tcols = kMaxThreads;
    p->tile_cols = int32_t(tcols);
    p->tile_rows = 1;
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
  p->max_segments = int32_t(segs);
  int64_t lg = (int64_t(p->tile_cols) - 1) / p->vec_group + 2;
  if (lg > num_groups) lg = num_groups;
  p->max_local_groups = int32_t(lg);
  p->workspace_bytes = uint64_t(blocks) * uint64_t(segs) * uint64_t(lg) * kAcc * sizeof(double);
  return KAT_OK;
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

// Kernel selection by (dtype, vec).
const void* fwd_kernel_for(int dtype, int vec) {
  switch (dtype) {
    case KAT_DTYPE_F32:
      switch (vec) {
        case 4: return (const void*)kat_fwd_kernel<float, 4, kUnroll>;
        case 2: return (const void*)kat_fwd_kernel<float, 2, kUnroll>;
        default: return (const void*)kat_fwd_kernel<float, 1, kUnroll>;
      }
    case KAT_DTYPE_F16:
      switch (vec) {
        case 8: return (const void*)kat_fwd_kernel<__half, 8, kUnroll>;
        case 4: return (const void*)kat_fwd_kernel<__half, 4, kUnroll>;
        case 2: return (const void*)kat_fwd_kernel<__half, 2, kUnroll>;
        default: return (const void*)kat_fwd_kernel<__half, 1, kUnroll>;
      }
    default:
      switch (vec) {
        case 8: return (const void*)kat_fwd_kernel<__nv_bfloat16, 8, kUnroll>;
        case 4: return (const void*)kat_fwd_kernel<__nv_bfloat16, 4, kUnroll>;
        case 2: return (const void*)kat_fwd_kernel<__nv_bfloat16, 2, kUnroll>;
        default: return (const void*)kat_fwd_kernel<__nv_bfloat16, 1, kUnroll>;
      }
  }
}

const void* bwd_kernel_for(int dtype, int vec) {
  switch (dtype) {
    case KAT_DTYPE_F32:
      switch (vec) {
        case 4: return (const void*)kat_bwd_kernel<float, 4, kUnroll>;
        case 2: return (const void*)kat_bwd_kernel<float, 2, kUnroll>;
        default: return (const void*)kat_bwd_kernel<float, 1, kUnroll>;
      }
    case KAT_DTYPE_F16:
      switch (vec) {
        case 8: return (const void*)kat_bwd_kernel<__half, 8, kUnroll>;
        case 4: return (const void*)kat_bwd_kernel<__half, 4, kUnroll>;
        case 2: return (const void*)kat_bwd_kernel<__half, 2, kUnroll>;
        default: return (const void*)kat_bwd_kernel<__half, 1, kUnroll>;
      }
    default:
      switch (vec) {
        case 8: return (const void*)kat_bwd_kernel<__nv_bfloat16, 8, kUnroll>;
        case 4: return (const void*)kat_bwd_kernel<__nv_bfloat16, 4, kUnroll>;
        case 2: return (const void*)kat_bwd_kernel<__nv_bfloat16, 2, kUnroll>;
        default: return (const void*)kat_bwd_kernel<__nv_bfloat16, 1, kUnroll>;
      }
  }
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

int plan_for_launch(const void* fn, int64_t batch, int64_t channels, int64_t inner,
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

template <typename Tio, int V>
cudaError_t launch_fwd_t(const void* x, void* y, const float* num, const float* den, const Plan& p,
                         cudaStream_t s) {
  kat_fwd_kernel<Tio, V, kUnroll><<<dim3(unsigned(p.blocks)), dim3(unsigned(p.threads)), 0, s>>>(
      static_cast<const Tio*>(x), static_cast<Tio*>(y), num, den, p);
  return cudaGetLastError();
}

template <typename Tio, int V>
cudaError_t launch_bwd_t(const void* x, const void* gy, void* dx, const float* num,
                         const float* den, double* partial, const Plan& p, cudaStream_t s) {
  kat_bwd_kernel<Tio, V, kUnroll><<<dim3(unsigned(p.blocks)), dim3(unsigned(p.threads)), 0, s>>>(
      static_cast<const Tio*>(x), static_cast<const Tio*>(gy), static_cast<Tio*>(dx), num, den,
      partial, p);
  return cudaGetLastError();
}

cudaError_t launch_fwd(int dtype, int vec, const void* x, void* y, const float* num,
                       const float* den, const Plan& p, cudaStream_t s) {
  switch (dtype) {
    case KAT_DTYPE_F32:
      if (vec == 4) return launch_fwd_t<float, 4>(x, y, num, den, p, s);
      if (vec == 2) return launch_fwd_t<float, 2>(x, y, num, den, p, s);
      return launch_fwd_t<float, 1>(x, y, num, den, p, s);
    case KAT_DTYPE_F16:
      if (vec == 8) return launch_fwd_t<__half, 8>(x, y, num, den, p, s);
      if (vec == 4) return launch_fwd_t<__half, 4>(x, y, num, den, p, s);
      if (vec == 2) return launch_fwd_t<__half, 2>(x, y, num, den, p, s);
      return launch_fwd_t<__half, 1>(x, y, num, den, p, s);
    default:
      if (vec == 8) return launch_fwd_t<__nv_bfloat16, 8>(x, y, num, den, p, s);
      if (vec == 4) return launch_fwd_t<__nv_bfloat16, 4>(x, y, num, den, p, s);
      if (vec == 2) return launch_fwd_t<__nv_bfloat16, 2>(x, y, num, den, p, s);
      return launch_fwd_t<__nv_bfloat16, 1>(x, y, num, den, p, s);
  }
}

cudaError_t launch_bwd(int dtype, int vec, const void* x, const void* gy, void* dx,
                       const float* num, const float* den, double* partial, const Plan& p,
                       cudaStream_t s) {
  switch (dtype) {
    case KAT_DTYPE_F32:
      if (vec == 4) return launch_bwd_t<float, 4>(x, gy, dx, num, den, partial, p, s);
      if (vec == 2) return launch_bwd_t<float, 2>(x, gy, dx, num, den, partial, p, s);
      return launch_bwd_t<float, 1>(x, gy, dx, num, den, partial, p, s);
    case KAT_DTYPE_F16:
      if (vec == 8) return launch_bwd_t<__half, 8>(x, gy, dx, num, den, partial, p, s);
      if (vec == 4) return launch_bwd_t<__half, 4>(x, gy, dx, num, den, partial, p, s);
      if (vec == 2) return launch_bwd_t<__half, 2>(x, gy, dx, num, den, partial, p, s);
      return launch_bwd_t<__half, 1>(x, gy, dx, num, den, partial, p, s);
    default:
      if (vec == 8) return launch_bwd_t<__nv_bfloat16, 8>(x, gy, dx, num, den, partial, p, s);
      if (vec == 4) return launch_bwd_t<__nv_bfloat16, 4>(x, gy, dx, num, den, partial, p, s);
      if (vec == 2) return launch_bwd_t<__nv_bfloat16, 2>(x, gy, dx, num, den, partial, p, s);
      return launch_bwd_t<__nv_bfloat16, 1>(x, gy, dx, num, den, partial, p, s);
  }
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
    default: return "unknown kat_rational status";
  }
}

int kat_rational_abi_version(void) { return KAT_RATIONAL_ABI_VERSION; }

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

int kat_rational_fwd(const void* x, void* y, const float* numerator, const float* denominator,
                     int64_t batch, int64_t channels, int64_t inner, int64_t num_groups, int dtype,
                     void* stream) {
  int64_t n = 0;
  int st = validate_dims(batch, channels, inner, num_groups, dtype, &n);
  if (st != KAT_OK) return st;
  if (numerator == nullptr || denominator == nullptr) return KAT_ERR_NULL_POINTER;
  if (n == 0) return KAT_OK;
  if (x == nullptr || y == nullptr) return KAT_ERR_NULL_POINTER;
  const int64_t gw = (channels / num_groups) * inner;
  const void* ptrs[2] = {x, y};
  const int vec = pick_vec(dtype, gw, ptrs, 2);
  Plan p;
  st = plan_for_launch(fwd_kernel_for(dtype, vec), batch, channels, inner, num_groups, dtype, vec,
                       &p);
  if (st != KAT_OK) return st;
  if (launch_fwd(dtype, vec, x, y, numerator, denominator, p,
                 static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return KAT_ERR_CUDA;
  return KAT_OK;
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
  for (int vec = max_vec_for(dtype); vec >= 1; vec >>= 1) {
    if (gw % vec != 0) continue;
    Plan p;
    st = plan_for_launch(bwd_kernel_for(dtype, vec), batch, channels, inner, num_groups, dtype, vec,
                         &p);
    if (st != KAT_OK) break;
    if (p.workspace_bytes > need) need = p.workspace_bytes;
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
  int64_t n = 0;
  int st = validate_dims(batch, channels, inner, num_groups, dtype, &n);
  if (st != KAT_OK) return st;
  if (numerator == nullptr || denominator == nullptr || grad_numerator == nullptr ||
      grad_denominator == nullptr)
    return KAT_ERR_NULL_POINTER;
  if (n != 0 && (x == nullptr || grad_out == nullptr)) return KAT_ERR_NULL_POINTER;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t gw = (channels / num_groups) * inner;
  const void* ptrs[3] = {x, grad_out, grad_x};
  const int vec = n == 0 ? 1 : pick_vec(dtype, gw, ptrs, 3);
  Plan p;
  if (n == 0) {
    st = make_plan_impl(batch, channels, inner, num_groups, dtype, vec, 1, 1, &p);
  } else {
    st = plan_for_launch(bwd_kernel_for(dtype, vec), batch, channels, inner, num_groups, dtype,
                         vec, &p);
  }
  if (st != KAT_OK) return st;
  if (p.blocks > 0) {
    if (workspace == nullptr || workspace_bytes < p.workspace_bytes ||
        (reinterpret_cast<uintptr_t>(workspace) % 16) != 0)
      return KAT_ERR_WORKSPACE;
    if (launch_bwd(dtype, vec, x, grad_out, grad_x, numerator, denominator,
                   static_cast<double*>(workspace), p, s) != cudaSuccess)
      return KAT_ERR_CUDA;
  }
  if (num_groups > 0x7fffffff) return KAT_ERR_BAD_GROUPS;
  kat_bwd_reduce_kernel<<<dim3(unsigned(num_groups)), dim3(kReduceThreads), 0, s>>>(
      static_cast<const double*>(workspace), denominator, grad_numerator, grad_denominator, p);
  if (cudaGetLastError() != cudaSuccess) return KAT_ERR_CUDA;
  return KAT_OK;
}

}  // extern "C"
