// kat_math.cuh — element codecs and the per-element rational math shared by the
// activation kernels (kat_rational.cu) and the GEMM kernels with a rational epilogue
// (kat_gemm.cu).  Included inside each translation unit's anonymous namespace.
//
// Formula (kat_rational/kat_1dgroup_torch.py:27-78 of the reference):
//   y = P(x) / Q(x),  P = sum_{k=0..5} a_k x^k,  Q = 1 + sum_{i=1..4} |b_i| x^i
// and the abs-after-sum variant Q = 1 + |sum_i b_i x^i| (rational_kat_cu/__init__.py:13-18).
// The includer provides <cuda_runtime.h>, <cuda_bf16.h>, <cuda_fp16.h>, <stdint.h> and
// kat_rational.h before opening its namespace.
#pragma once

constexpr int kAcc = 10;          // 6 numerator + 4 denominator gradient sums

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
  // Byte permutes run on the integer ALU, keeping the FMA pipe for the arithmetic.
  __device__ __forceinline__ static float2 unpack_word(uint32_t w) {
    return make_float2(__uint_as_float(__byte_perm(w, 0u, 0x1044u)),
                       __uint_as_float(__byte_perm(w, 0u, 0x3244u)));
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

// Read-only streaming load; 16-byte vectors skip L1 and ask L2 for 256-byte fetches.
template <typename Tio, int V>
__device__ __forceinline__ typename RawOf<Tio, V>::T load_raw(const Tio* __restrict__ ptr) {
  using B = typename RawOf<Tio, V>::T;
  if constexpr (sizeof(B) == 16) {
    uint4 v;
    asm("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0, %1, %2, %3}, [%4];"
        : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
        : "l"(ptr));
    return v;
  } else if constexpr (sizeof(B) == 2) {
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

// Two elements computed with scalar fp32 instructions (the fp32 backward: measured faster
// there than the paired instructions, while 16-bit inputs gain from pairing).
struct S2 {
  float x, y;
};
__device__ __forceinline__ S2 fma_(S2 a, S2 b, S2 c) {
  return S2{__fmaf_rn(a.x, b.x, c.x), __fmaf_rn(a.y, b.y, c.y)};
}
__device__ __forceinline__ S2 mul_(S2 a, S2 b) { return S2{__fmul_rn(a.x, b.x), __fmul_rn(a.y, b.y)}; }
__device__ __forceinline__ S2 add_(S2 a, S2 b) { return S2{__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y)}; }
__device__ __forceinline__ S2 neg_(S2 a) { return S2{-a.x, -a.y}; }
__device__ __forceinline__ S2 rcp_(S2 q) { return S2{rcp_(q.x), rcp_(q.y)}; }
template <> __device__ __forceinline__ S2 bcast<S2>(float v) { return S2{v, v}; }
__device__ __forceinline__ float lane_sum(S2 v) { return v.x + v.y; }

// Pair <-> lane type.
template <typename L> __device__ __forceinline__ L to_lane(float2 v);
template <> __device__ __forceinline__ float2 to_lane<float2>(float2 v) { return v; }
template <> __device__ __forceinline__ S2 to_lane<S2>(float2 v) { return S2{v.x, v.y}; }
__device__ __forceinline__ float2 from_lane(float2 v) { return v; }
__device__ __forceinline__ float2 from_lane(S2 v) { return make_float2(v.x, v.y); }

// Coefficients of one group, broadcast to the lane type.
template <typename L> struct FwdCoef {
  L a0, a1, a2, a3, a4, a5;  // numerator
  L c1, c2, c3, c4;          // |b_i|
  L one;
};

template <typename L> struct BwdCoef {
  L a0, a1, a2, a3, a4, a5;  // numerator
  L c1, c2, c3, c4;          // |b_i|
  L one;
};

// Denominator formulas.  kFormulaKat: Q = 1 + sum_i |b_i| x^i (coefficients made
// non-negative once, kat_rational/kat_1dgroup_torch.py:63-69).  kFormulaAbsSum:
// Q = 1 + |D(x)|, D = sum_i b_i x^i with raw coefficients and the absolute value taken after
// the sum (rational_kat_cu/__init__.py:13-18, kat_rational/rational_triton.py:65-72).
constexpr int kFormulaKat = KAT_FORMULA_KAT;
constexpr int kFormulaAbsSum = KAT_FORMULA_ABS_SUM;

template <int kF>
__device__ __forceinline__ float den_coef(const float* b, int i) {
  return kF == kFormulaKat ? fabsf(__ldg(b + i)) : __ldg(b + i);
}

template <typename L, int kF>
__device__ __forceinline__ void load_fwd_coef(const float* __restrict__ num,
                                              const float* __restrict__ den, int64_t g,
                                              FwdCoef<L>& c, int num_stride = 6) {
  const float* a = num + g * num_stride;   // num_stride 0: one numerator row for every group
  const float* b = den + g * 4;
  c.a0 = bcast<L>(__ldg(a + 0)); c.a1 = bcast<L>(__ldg(a + 1)); c.a2 = bcast<L>(__ldg(a + 2));
  c.a3 = bcast<L>(__ldg(a + 3)); c.a4 = bcast<L>(__ldg(a + 4)); c.a5 = bcast<L>(__ldg(a + 5));
  c.c1 = bcast<L>(den_coef<kF>(b, 0)); c.c2 = bcast<L>(den_coef<kF>(b, 1));
  c.c3 = bcast<L>(den_coef<kF>(b, 2)); c.c4 = bcast<L>(den_coef<kF>(b, 3));
  c.one = bcast<L>(1.0f);
}

template <typename L, int kF>
__device__ __forceinline__ void load_bwd_coef(const float* __restrict__ num,
                                              const float* __restrict__ den, int64_t g,
                                              BwdCoef<L>& c, int num_stride = 6) {
  const float* a = num + g * num_stride;   // num_stride 0: one numerator row for every group
  const float* b = den + g * 4;
  c.a0 = bcast<L>(__ldg(a + 0)); c.a1 = bcast<L>(__ldg(a + 1)); c.a2 = bcast<L>(__ldg(a + 2));
  c.a3 = bcast<L>(__ldg(a + 3)); c.a4 = bcast<L>(__ldg(a + 4)); c.a5 = bcast<L>(__ldg(a + 5));
  c.c1 = bcast<L>(den_coef<kF>(b, 0)); c.c2 = bcast<L>(den_coef<kF>(b, 1));
  c.c3 = bcast<L>(den_coef<kF>(b, 2)); c.c4 = bcast<L>(den_coef<kF>(b, 3));
  c.one = bcast<L>(1.0f);
}

// |v| and v with its sign flipped where s < 0 (s = -0 counts as non-negative, as the
// reference's where(D < 0, -1, 1)).
__device__ __forceinline__ float abs_(float v) { return fabsf(v); }
__device__ __forceinline__ float2 abs_(float2 v) { return make_float2(fabsf(v.x), fabsf(v.y)); }
__device__ __forceinline__ float flip_neg_(float v, float s) { return s < 0.0f ? -v : v; }
__device__ __forceinline__ float2 flip_neg_(float2 v, float2 s) {
  return make_float2(flip_neg_(v.x, s.x), flip_neg_(v.y, s.y));
}
__device__ __forceinline__ S2 abs_(S2 v) { return S2{fabsf(v.x), fabsf(v.y)}; }
__device__ __forceinline__ S2 flip_neg_(S2 v, S2 s) {
  return S2{flip_neg_(v.x, s.x), flip_neg_(v.y, s.y)};
}

// Forward on one lane (scalar or pair).
template <typename L, bool kExactDiv, int kF>
__device__ __forceinline__ L fwd_math(L x, const FwdCoef<L>& c) {
  L p = fma_(c.a5, x, c.a4);
  p = fma_(p, x, c.a3);
  p = fma_(p, x, c.a2);
  p = fma_(p, x, c.a1);
  p = fma_(p, x, c.a0);
  L q = fma_(c.c4, x, c.c3);
  q = fma_(q, x, c.c2);
  q = fma_(q, x, c.c1);
  if constexpr (kF == kFormulaKat) {
    q = fma_(q, x, c.one);
  } else {
    q = add_(abs_(mul_(q, x)), c.one);  // 1 + |D|, D = (Horner of b3..b0) * x
  }
  if constexpr (kExactDiv) {
    return div_rn_(p, q);
  } else {
    return mul_(p, rcp_(q));
  }
}

// Backward on one lane: returns dx and adds this lane's gradient terms into
// acc[0..5] (sum u x^k) and acc[6..9] (sum u y x^i, i = 1..4).
template <typename L, bool kRefine, int kF>
__device__ __forceinline__ L bwd_math(L x, L go, const BwdCoef<L>& c, L (&acc)[kAcc]) {
  // Horner for P and Q; the derivatives come from the same partial sums
  // (d_k = d_{k+1} x + p_{k+1}), so no scaled coefficients are needed.
  L p = fma_(c.a5, x, c.a4);
  L dp = fma_(c.a5, x, p);
  p = fma_(p, x, c.a3);
  dp = fma_(dp, x, p);
  p = fma_(p, x, c.a2);
  dp = fma_(dp, x, p);
  p = fma_(p, x, c.a1);
  dp = fma_(dp, x, p);
  p = fma_(p, x, c.a0);
  L q = fma_(c.c4, x, c.c3);
  L dq = fma_(c.c4, x, q);
  q = fma_(q, x, c.c2);
  dq = fma_(dq, x, q);
  q = fma_(q, x, c.c1);
  dq = fma_(dq, x, q);
  L d_sign;  // abs-after-sum: D, whose sign flips Q' and the denominator gradient terms
  if constexpr (kF == kFormulaKat) {
    q = fma_(q, x, c.one);
  } else {
    // Here q = h(x) = D / x (the Horner value before its last step) and dq = D' (the
    // derivative recurrence has run to its end): D = h x, Q = 1 + |D|, Q' = sgn(D) D'.
    d_sign = mul_(q, x);
    dq = flip_neg_(dq, d_sign);
    q = add_(abs_(d_sign), c.one);
  }
  const L x2 = mul_(x, x);
  L r = rcp_(q);
  if constexpr (kRefine) {  // Newton-Raphson: r <- r + r (1 - q r)
    const L e = fma_(neg_(q), r, c.one);
    r = fma_(r, e, r);
  }
  const L u = mul_(go, r);            // go / Q
  const L y = mul_(p, r);             // P / Q
  const L t = fma_(neg_(y), dq, dp);  // P' - y Q'
  L w = mul_(u, y);                   // go P / Q^2
  if constexpr (kF != kFormulaKat) w = flip_neg_(w, d_sign);  // sgn(D) go P / Q^2
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
template <typename Tio, int V, typename L, bool kExact, int kF = kFormulaKat>
__device__ __forceinline__ typename RawOf<Tio, V>::T fwd_vec(typename RawOf<Tio, V>::T raw,
                                                             const FwdCoef<L>& c) {
  Frag<V> f = unpack<Tio, V>(raw);
  if constexpr (V == 1) {
    f.s = fwd_math<float, kExact, kF>(f.s, c);
  } else {
#pragma unroll
    for (int k = 0; k < V / 2; ++k) f.p[k] = fwd_math<float2, kExact, kF>(f.p[k], c);
  }
  return pack<Tio, V>(f);
}

template <typename Tio, int V, typename L, bool kRefine, int kF = kFormulaKat>
__device__ __forceinline__ typename RawOf<Tio, V>::T bwd_vec(typename RawOf<Tio, V>::T rx,
                                                             typename RawOf<Tio, V>::T rg,
                                                             const BwdCoef<L>& c,
                                                             L (&acc)[kAcc]) {
  Frag<V> fx = unpack<Tio, V>(rx);
  const Frag<V> fg = unpack<Tio, V>(rg);
  if constexpr (V == 1) {
    fx.s = bwd_math<float, kRefine, kF>(fx.s, fg.s, c, acc);
  } else {
#pragma unroll
    for (int k = 0; k < V / 2; ++k)
      fx.p[k] = from_lane(bwd_math<L, kRefine, kF>(to_lane<L>(fx.p[k]), to_lane<L>(fg.p[k]), c, acc));
  }
  return pack<Tio, V>(fx);
}
