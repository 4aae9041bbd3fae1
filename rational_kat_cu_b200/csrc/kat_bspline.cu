// B-spline basis (Cox-de Boor) forward and backward for sm_100a: the basis evaluation of
// efficient-KAN layers that the reference fuses in rational_kat_cu/bspline_basis.py.
//
// One thread per input element x[b, d].  Instead of running the recursion over every knot
// interval (the reference evaluates all n_knots - 1 indicators and every level in full), a
// thread finds the one interval t_i <= x < t_{i+1} by binary search on its channel's knots and
// evaluates only the triangle of values that can be non-zero there (k + 1 values at level k),
// each term with the reference's operation order — ((x - t_j) / max(t_{j+k} - t_j, 1e-8)) times
// the lower-order value, the two terms added, no fused multiply-add — so the non-zero values
// match the full recursion bit for bit and every other basis value is zero, as there.
// Outputs (forward) and incoming gradients (backward) move through shared memory so each
// block reads and writes its contiguous [elements x n_basis] slab with coalesced accesses.
//
// Knots must be non-decreasing along each channel (KANLinear's grid and update_grid produce
// such grids).  A non-finite x gives NaN in every basis value, as the reference's full
// recursion does (its 0 * inf terms).

#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "kat_bspline.h"
#include "kat_rational.h"

namespace {

constexpr int kBsThreads = 256;
constexpr int kMaxOrder = 5;
constexpr int kMaxKnots = 64;
constexpr float kEps = 1e-8f;

// Largest i in [0, n - 2] with t[i] <= x, for t[0] <= x < t[n - 1] (non-decreasing t).
__device__ __forceinline__ int find_span(const float* __restrict__ t, int n, float x) {
  int lo = 0, hi = n - 1;  // invariant: t[lo] <= x < t[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (__ldg(t + mid) <= x) lo = mid; else hi = mid;
  }
  return lo;
}

// Knots t[i - kOrder .. i + kOrder + 1] of span i in registers (indices outside [0, n - 1] are
// clamped: those entries are never used, see span_basis).
template <int kOrder>
__device__ __forceinline__ void load_window(const float* __restrict__ t, int n, int i,
                                            float (&w)[2 * kOrder + 2]) {
#pragma unroll
  for (int q = 0; q < 2 * kOrder + 2; ++q) {
    const int j = min(max(i - kOrder + q, 0), n - 1);
    w[q] = __ldg(t + j);
  }
}

// Basis values of order kOrder that can be non-zero at x in span i: b[m] = B^kOrder_{i-kOrder+m}
// for m = 0..kOrder (entries whose index is outside [0, n - 2 - kOrder] are left 0), and,
// when kGrad, their derivatives db[m].  Level by level, as the recursion runs; knot t_j is
// w[j - i + kOrder].
template <int kOrder, bool kGrad>
__device__ __forceinline__ void span_basis(const float (&w)[2 * kOrder + 2], int n, int i,
                                           float x, float (&b)[kMaxOrder + 1],
                                           float (&db)[kMaxOrder + 1]) {
  float prev[kMaxOrder + 1], dprev[kMaxOrder + 1];
  prev[0] = 1.0f;
  dprev[0] = 0.0f;
#pragma unroll
  for (int k = 1; k <= kOrder; ++k) {
#pragma unroll
    for (int m = 0; m <= k; ++m) {
      const int j = i - k + m;
      const int o = kOrder - k + m;  // position of t_j in the window
      float v = 0.0f, dv = 0.0f;
      if (j >= 0 && j <= n - 2 - k) {
        // left term: (x - t_j) / max(t_{j+k} - t_j, eps) * B^{k-1}_j   (prev index m - 1)
        float left = 0.0f, dleft = 0.0f;
        if (m >= 1) {
          const float d1 = fmaxf(__fsub_rn(w[o + k], w[o]), kEps);
          const float u = __fdiv_rn(__fsub_rn(x, w[o]), d1);
          left = __fmul_rn(u, prev[m - 1]);
          if constexpr (kGrad)
            dleft = __fadd_rn(__fdiv_rn(prev[m - 1], d1), __fmul_rn(u, dprev[m - 1]));
        }
        // right term: (t_{j+k+1} - x) / max(t_{j+k+1} - t_{j+1}, eps) * B^{k-1}_{j+1}   (m)
        float right = 0.0f, dright = 0.0f;
        if (m <= k - 1) {
          const float d2 = fmaxf(__fsub_rn(w[o + k + 1], w[o + 1]), kEps);
          const float r = __fdiv_rn(__fsub_rn(w[o + k + 1], x), d2);
          right = __fmul_rn(r, prev[m]);
          if constexpr (kGrad)
            dright = __fsub_rn(__fmul_rn(r, dprev[m]), __fdiv_rn(prev[m], d2));
        }
        v = __fadd_rn(left, right);
        if constexpr (kGrad) dv = __fadd_rn(dleft, dright);
      }
      b[m] = v;
      db[m] = dv;
    }
#pragma unroll
    for (int m = 0; m <= k; ++m) {
      prev[m] = b[m];
      dprev[m] = db[m];
    }
  }
}

// Channel of element e0 + threadIdx.x, given d0 = e0 % features (one division per block).
__device__ __forceinline__ int64_t channel_of(int64_t d0, int64_t features) {
  int64_t d = d0 + threadIdx.x;
  if (features >= blockDim.x) return d >= features ? d - features : d;
  return d % features;
}

// Copies `count` floats between global memory and the block's slab with 16-byte accesses
// when both sides are 16-byte aligned (the slab always is; the global side is when the
// block's first float is), scalar otherwise.
template <bool kToGlobal>
__device__ __forceinline__ void copy_slab(float* __restrict__ slab, float* __restrict__ g,
                                          int count) {
  if ((reinterpret_cast<uintptr_t>(g) & 15) == 0) {
    const int c4 = count >> 2;
    float4* s4 = reinterpret_cast<float4*>(slab);
    float4* g4 = reinterpret_cast<float4*>(g);
#pragma unroll 4
    for (int q = threadIdx.x; q < c4; q += kBsThreads) {
      if constexpr (kToGlobal) g4[q] = s4[q]; else s4[q] = __ldg(g4 + q);
    }
    for (int q = (c4 << 2) + threadIdx.x; q < count; q += kBsThreads) {
      if constexpr (kToGlobal) g[q] = slab[q]; else slab[q] = __ldg(g + q);
    }
  } else {
#pragma unroll 4
    for (int q = threadIdx.x; q < count; q += kBsThreads) {
      if constexpr (kToGlobal) g[q] = slab[q]; else slab[q] = __ldg(g + q);
    }
  }
}

template <int kOrder>
__global__ void __launch_bounds__(kBsThreads)
kat_bspline_fwd_kernel(const float* __restrict__ x, const float* __restrict__ grid,
                       float* __restrict__ out, int64_t n_elem, int64_t features, int n_knots) {
  extern __shared__ __align__(16) float slab[];  // [kBsThreads][n_basis]
  __shared__ int64_t s_d0;
  const int nb = n_knots - 1 - kOrder;
  const int64_t e0 = int64_t(blockIdx.x) * kBsThreads;
  const int count = int(min(int64_t(kBsThreads), n_elem - e0)) * nb;
  if (threadIdx.x == 0) s_d0 = e0 % features;
  {
    float4* s4 = reinterpret_cast<float4*>(slab);
    const int c4 = (kBsThreads * nb + 3) >> 2;
    for (int q = threadIdx.x; q < c4; q += kBsThreads) s4[q] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  __syncthreads();
  const int64_t e = e0 + threadIdx.x;
  if (e < n_elem) {
    const float v = x[e];
    const float* t = grid + channel_of(s_d0, features) * n_knots;
    float* row = slab + threadIdx.x * nb;
    if (!isfinite(v)) {
      for (int j = 0; j < nb; ++j) row[j] = __int_as_float(0x7fc00000);
    } else if (v >= __ldg(t) && v < __ldg(t + n_knots - 1)) {
      const int i = find_span(t, n_knots, v);
      float w[2 * kOrder + 2];
      load_window<kOrder>(t, n_knots, i, w);
      float b[kMaxOrder + 1], db[kMaxOrder + 1];
      span_basis<kOrder, false>(w, n_knots, i, v, b, db);
#pragma unroll
      for (int m = 0; m <= kOrder; ++m) {
        const int j = i - kOrder + m;
        if (j >= 0 && j < nb) row[j] = b[m];
      }
    }
  }
  __syncthreads();
  copy_slab<true>(slab, out + e0 * nb, count);
}

template <int kOrder>
__global__ void __launch_bounds__(kBsThreads)
kat_bspline_bwd_kernel(const float* __restrict__ x, const float* __restrict__ grid,
                       const float* __restrict__ gb, float* __restrict__ gx, int64_t n_elem,
                       int64_t features, int n_knots) {
  extern __shared__ __align__(16) float slab[];  // [kBsThreads][n_basis]
  __shared__ int64_t s_d0;
  const int nb = n_knots - 1 - kOrder;
  const int64_t e0 = int64_t(blockIdx.x) * kBsThreads;
  const int count = int(min(int64_t(kBsThreads), n_elem - e0)) * nb;
  if (threadIdx.x == 0) s_d0 = e0 % features;
  copy_slab<false>(slab, const_cast<float*>(gb) + e0 * nb, count);
  __syncthreads();
  const int64_t e = e0 + threadIdx.x;
  if (e >= n_elem) return;
  const float v = x[e];
  const float* row = slab + threadIdx.x * nb;
  float acc = 0.0f;
  const float* t = grid + channel_of(s_d0, features) * n_knots;
  if (!isfinite(v)) {
    acc = __int_as_float(0x7fc00000);
  } else if (v >= __ldg(t) && v < __ldg(t + n_knots - 1)) {
    const int i = find_span(t, n_knots, v);
    float w[2 * kOrder + 2];
    load_window<kOrder>(t, n_knots, i, w);
    float b[kMaxOrder + 1], db[kMaxOrder + 1];
    span_basis<kOrder, true>(w, n_knots, i, v, b, db);
#pragma unroll
    for (int m = 0; m <= kOrder; ++m) {
      const int j = i - kOrder + m;
      if (j >= 0 && j < nb) acc = __fadd_rn(acc, __fmul_rn(row[j], db[m]));
    }
  }
  gx[e] = acc;
}

int validate(int64_t batch, int64_t features, int32_t n_knots, int32_t order, int64_t* n) {
  if (batch < 0 || features < 0) return KAT_ERR_BAD_SHAPE;
  if (order < 1 || order > kMaxOrder || n_knots < order + 2 || n_knots > kMaxKnots)
    return KAT_ERR_BAD_SHAPE;
  if (features != 0 && batch > (int64_t(1) << 40) / features) return KAT_ERR_BAD_SHAPE;
  *n = batch * features;
  return KAT_OK;
}

template <int kOrder>
cudaError_t launch_fwd(const float* x, const float* grid, float* out, int64_t n, int64_t f,
                       int nk, cudaStream_t s) {
  const size_t smem = size_t(kBsThreads) * (nk - 1 - kOrder) * sizeof(float);
  if (smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute((const void*)kat_bspline_fwd_kernel<kOrder>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               int(smem));
    if (e != cudaSuccess) return e;
  }
  const unsigned blocks = unsigned((n + kBsThreads - 1) / kBsThreads);
  kat_bspline_fwd_kernel<kOrder><<<blocks, kBsThreads, smem, s>>>(x, grid, out, n, f, nk);
  return cudaGetLastError();
}

template <int kOrder>
cudaError_t launch_bwd(const float* x, const float* grid, const float* gb, float* gx, int64_t n,
                       int64_t f, int nk, cudaStream_t s) {
  const size_t smem = size_t(kBsThreads) * (nk - 1 - kOrder) * sizeof(float);
  if (smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute((const void*)kat_bspline_bwd_kernel<kOrder>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               int(smem));
    if (e != cudaSuccess) return e;
  }
  const unsigned blocks = unsigned((n + kBsThreads - 1) / kBsThreads);
  kat_bspline_bwd_kernel<kOrder><<<blocks, kBsThreads, smem, s>>>(x, grid, gb, gx, n, f, nk);
  return cudaGetLastError();
}

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
    case 1: e = launch_fwd<1>(x, grid, bases, n, features, n_knots, s); break;
    case 2: e = launch_fwd<2>(x, grid, bases, n, features, n_knots, s); break;
    case 3: e = launch_fwd<3>(x, grid, bases, n, features, n_knots, s); break;
    case 4: e = launch_fwd<4>(x, grid, bases, n, features, n_knots, s); break;
    default: e = launch_fwd<5>(x, grid, bases, n, features, n_knots, s); break;
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
    case 1: e = launch_bwd<1>(x, grid, grad_bases, grad_x, n, features, n_knots, s); break;
    case 2: e = launch_bwd<2>(x, grid, grad_bases, grad_x, n, features, n_knots, s); break;
    case 3: e = launch_bwd<3>(x, grid, grad_bases, grad_x, n, features, n_knots, s); break;
    case 4: e = launch_bwd<4>(x, grid, grad_bases, grad_x, n, features, n_knots, s); break;
    default: e = launch_bwd<5>(x, grid, grad_bases, grad_x, n, features, n_knots, s); break;
  }
  return e == cudaSuccess ? KAT_OK : KAT_ERR_CUDA;
}

}  // extern "C"
