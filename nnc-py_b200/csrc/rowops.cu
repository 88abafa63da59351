// Row-wise operators: softmax, layernorm, reducemean / reducesum.
//
// All three decompose the tensor as [outer, dim, inner] around `axis` exactly
// like the reference (ops.c:260-310, :2095-2171, :1892-1989).
//   inner == 1 : rows of at most 1024 elements take one warp per row (the
//                row in registers, shuffle reductions only); longer rows one
//                128-thread block per row with the row cached in shared
//                memory (up to 32768 elements; beyond that, one 256-thread
//                block per row re-reading it). Every element is read once and
//                written once — 8 bytes of HBM traffic per element.
//   inner  > 1 : one thread per (outer, inner) column walking `dim` with
//                stride `inner`; consecutive threads read consecutive
//                addresses, so every pass is coalesced.
// Reduce accumulates in fp64 (the reference: Kahan-compensated fp32).
// Softmax and layernorm (reference: sequential fp32) sum each lane's values
// pairwise (warp kernels) or compensated (block kernels) in fp32 and combine
// the lanes in fp64, and scale by a reciprocal instead of dividing each
// element: results agree with the reference to within a few fp32 ulps.
#include <math.h>

#include "common.cuh"

namespace nnc {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxVPT = 32;  // registers per thread for a cached row (8192 floats)

__device__ __forceinline__ double warp_sum(double v) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Compensated fp32 accumulation (Neumaier): s + c carries the running sum
// to about one fp32 ulp whatever the count, at full fp32 rate; the lanes'
// (s + c) are then combined in fp64.
__device__ __forceinline__ void comp_add(float& s, float& c, float x) {
  const float t = __fadd_rn(s, x);
  const float e = fabsf(s) >= fabsf(x) ? __fadd_rn(__fsub_rn(s, t), x) : __fadd_rn(__fsub_rn(x, t), s);
  c = __fadd_rn(c, e);
  s = t;
}

// Pairwise (tree) fp32 sum of a lane's N values: error O(log2 N) ulps of
// the magnitudes summed, one add per value.
template <int N>
__device__ __forceinline__ float tree_sum(const float (&x)[N]) {
  float t[N];
#pragma unroll
  for (int k = 0; k < N; ++k) t[k] = x[k];
#pragma unroll
  for (int w = 1; w < N; w *= 2)
#pragma unroll
    for (int k = 0; k + w < N; k += 2 * w) t[k] = __fadd_rn(t[k], t[k + w]);
  return t[0];
}

// Element k of a lane's VPT values in a warp-per-row kernel: lane-strided
// scalars, or (VEC) float4 runs 4 lane + 128 (k / 4) + {0..3}.
template <bool VEC>
__device__ __forceinline__ int row_index(int lane, int k) {
  return VEC ? 128 * (k >> 2) + 4 * lane + (k & 3) : lane + 32 * k;
}

// Block-wide reductions for kThreads threads; `red` holds kThreads/32 slots.
__device__ double block_sum(double v, double* red) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  double t = (threadIdx.x < kThreads / 32) ? red[threadIdx.x] : 0.0;
  if (wid == 0) t = warp_sum(t);
  if (threadIdx.x == 0) red[0] = t;
  __syncthreads();
  return red[0];
}
__device__ float block_max(float v, float* red) {
  v = warp_max(v);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float t = (threadIdx.x < kThreads / 32) ? red[threadIdx.x] : -INFINITY;
  if (wid == 0) t = warp_max(t);
  if (threadIdx.x == 0) red[0] = t;
  __syncthreads();
  return red[0];
}

// ---------------------------------------------------------------- softmax --
// Row kernel: per row max, sum of expf(x - max), out = expf(x - max) / sum
// (ops.c:283-307). Values cached in registers when dim <= kThreads*kMaxVPT.
__global__ void __launch_bounds__(kThreads) softmax_row_kernel(const float* __restrict__ in,
                                                               float* __restrict__ out,
                                                               int64_t rows, int64_t dim) {
  __shared__ double red_d[kThreads / 32];
  __shared__ float red_f[kThreads / 32];
  const bool cached = dim <= (int64_t)kThreads * kMaxVPT;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const float* x = in + row * dim;
    float* y = out + row * dim;
    float v[kMaxVPT];
    float m = -INFINITY;
    if (cached) {
#pragma unroll
      for (int k = 0; k < kMaxVPT; ++k) {
        const int64_t i = threadIdx.x + (int64_t)k * kThreads;
        v[k] = (i < dim) ? x[i] : -INFINITY;
        m = (v[k] > m) ? v[k] : m;
      }
    } else {
      for (int64_t i = threadIdx.x; i < dim; i += kThreads) m = (x[i] > m) ? x[i] : m;
    }
    m = block_max(m, red_f);
    double s = 0.0;
    if (cached) {
#pragma unroll
      for (int k = 0; k < kMaxVPT; ++k) {
        const int64_t i = threadIdx.x + (int64_t)k * kThreads;
        if (i < dim) {
          v[k] = expf(v[k] - m);
          s += (double)v[k];
        }
      }
    } else {
      for (int64_t i = threadIdx.x; i < dim; i += kThreads) s += (double)expf(x[i] - m);
    }
    const float sum = (float)block_sum(s, red_d);
    if (cached) {
#pragma unroll
      for (int k = 0; k < kMaxVPT; ++k) {
        const int64_t i = threadIdx.x + (int64_t)k * kThreads;
        if (i < dim) y[i] = __fdiv_rn(v[k], sum);
      }
    } else {
      for (int64_t i = threadIdx.x; i < dim; i += kThreads) y[i] = __fdiv_rn(expf(x[i] - m), sum);
    }
  }
}

// Short rows (dim <= 32 VPT): one warp per row, VPT values per lane in
// registers (VEC: 16-byte loads and stores), shuffle reductions only; 8 rows
// per 256-thread block. The sum is a pairwise fp32 sum per lane, combined in
// fp64; outputs are e * (1 / sum) (within one ulp of e / sum).
template <int VPT, bool VEC>
__global__ void __launch_bounds__(kThreads, VPT <= 8 ? 4 : 2) softmax_warp_kernel(const float* __restrict__ in,
                                                                float* __restrict__ out,
                                                                int64_t rows, int dim) {
  static_assert(!VEC || VPT % 4 == 0, "vector rows hold whole float4 runs");
  const int lane = threadIdx.x & 31;
  const int64_t step = (int64_t)gridDim.x * (kThreads / 32);
  auto load_row = [&](int64_t row, float (&v)[VPT]) {
    const float* x = in + row * dim;
    if constexpr (VEC) {
#pragma unroll
      for (int k = 0; k < VPT; k += 4) {
        const int i = row_index<true>(lane, k);
        float4 t = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
        if (i < dim) t = __ldg(reinterpret_cast<const float4*>(x + i));
        v[k] = t.x; v[k + 1] = t.y; v[k + 2] = t.z; v[k + 3] = t.w;
      }
    } else {
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        const int i = row_index<false>(lane, k);
        v[k] = i < dim ? x[i] : -INFINITY;
      }
    }
  };
  // Short rows keep the next row's loads in flight while this row reduces.
  constexpr bool kPrefetch = VPT <= 8;
  int64_t row = (int64_t)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5);
  float vn[VPT];
  if (kPrefetch && row < rows) load_row(row, vn);
  for (; row < rows; row += step) {
    float* y = out + row * dim;
    float v[VPT];
    if constexpr (kPrefetch) {
#pragma unroll
      for (int k = 0; k < VPT; ++k) v[k] = vn[k];
      if (row + step < rows) load_row(row + step, vn);
    } else {
      load_row(row, v);
    }
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < VPT; ++k) m = (v[k] > m) ? v[k] : m;
    m = warp_max(m);
#pragma unroll
    for (int k = 0; k < VPT; ++k) v[k] = row_index<VEC>(lane, k) < dim ? expf(v[k] - m) : 0.0f;
    const float inv = __frcp_rn((float)warp_sum((double)tree_sum(v)));
    if constexpr (VEC) {
#pragma unroll
      for (int k = 0; k < VPT; k += 4) {
        const int i = row_index<true>(lane, k);
        if (i < dim)
          *reinterpret_cast<float4*>(y + i) =
              make_float4(__fmul_rn(v[k], inv), __fmul_rn(v[k + 1], inv), __fmul_rn(v[k + 2], inv),
                          __fmul_rn(v[k + 3], inv));
      }
    } else {
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        const int i = row_index<false>(lane, k);
        if (i < dim) y[i] = __fmul_rn(v[k], inv);
      }
    }
  }
}

// Long rows (dim <= kSmemRowMax): one 128-thread block per row with the row
// cached in shared memory (dynamic, dim floats), so many rows are in flight
// per SM; 16-byte accesses when dim % 4 == 0 and the bases are aligned.
constexpr int kRowThreads = 128;
constexpr int kSmemRowMax = 32768;  // 128 KB of shared memory
__device__ double block_sum128(double v, double* red) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  return red[0] + red[1] + red[2] + red[3];
}
__device__ float block_max128(float v, float* red) {
  v = warp_max(v);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  const float a = red[0] > red[1] ? red[0] : red[1];
  const float b = red[2] > red[3] ? red[2] : red[3];
  return a > b ? a : b;
}
__global__ void __launch_bounds__(kRowThreads) softmax_smem_kernel(const float* __restrict__ in,
                                                                   float* __restrict__ out,
                                                                   int64_t rows, int dim) {
  extern __shared__ __align__(16) float rowbuf[];
  __shared__ double red_d[4];
  __shared__ float red_f[4];
  const bool vec = (dim & 3) == 0 && ((((uintptr_t)in) | ((uintptr_t)out)) & 15) == 0;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const float* x = in + row * dim;
    float* y = out + row * dim;
    float m = -INFINITY;
    if (vec) {
      for (int i = threadIdx.x; i < dim / 4; i += kRowThreads) {
        const float4 t = reinterpret_cast<const float4*>(x)[i];
        reinterpret_cast<float4*>(rowbuf)[i] = t;
        m = (t.x > m) ? t.x : m;
        m = (t.y > m) ? t.y : m;
        m = (t.z > m) ? t.z : m;
        m = (t.w > m) ? t.w : m;
      }
    } else {
      for (int i = threadIdx.x; i < dim; i += kRowThreads) {
        const float t = x[i];
        rowbuf[i] = t;
        m = (t > m) ? t : m;
      }
    }
    m = block_max128(m, red_f);
    float s = 0.0f, c = 0.0f;
    for (int i = threadIdx.x; i < dim; i += kRowThreads) {
      const float e = expf(rowbuf[i] - m);
      rowbuf[i] = e;
      comp_add(s, c, e);
    }
    const float inv = __frcp_rn((float)block_sum128((double)s + (double)c, red_d));
    if (vec) {
      for (int i = threadIdx.x; i < dim / 4; i += kRowThreads) {
        const float4 e = reinterpret_cast<const float4*>(rowbuf)[i];
        reinterpret_cast<float4*>(y)[i] =
            make_float4(__fmul_rn(e.x, inv), __fmul_rn(e.y, inv), __fmul_rn(e.z, inv), __fmul_rn(e.w, inv));
      }
    } else {
      for (int i = threadIdx.x; i < dim; i += kRowThreads) y[i] = __fmul_rn(rowbuf[i], inv);
    }
    __syncthreads();  // rowbuf is reused by the next row
  }
}

// Strided kernel (inner > 1): one thread per (outer, inner) column.
__global__ void __launch_bounds__(kThreads) softmax_col_kernel(const float* __restrict__ in,
                                                               float* __restrict__ out,
                                                               int64_t outer, int64_t dim,
                                                               int64_t inner) {
  const int64_t cols = outer * inner;
  for (int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c < cols;
       c += (int64_t)gridDim.x * blockDim.x) {
    const int64_t o = c / inner, j = c % inner;
    const float* x = in + o * dim * inner + j;
    float* y = out + o * dim * inner + j;
    float m = -INFINITY;
    for (int64_t s = 0; s < dim; ++s) m = (x[s * inner] > m) ? x[s * inner] : m;
    double acc = 0.0;
    for (int64_t s = 0; s < dim; ++s) acc += (double)expf(x[s * inner] - m);
    const float sum = (float)acc;
    for (int64_t s = 0; s < dim; ++s) y[s * inner] = __fdiv_rn(expf(x[s * inner] - m), sum);
  }
}

// -------------------------------------------------------------- layernorm --
// Normalises each [norm, inner] slab (ops.c:2130-2168): mean, variance of
// (x - mean), std = sqrtf(var + eps), y = scale[i] * ((x - mean) / std) + bias[i]
// with scale/bias indexed by the axis coordinate i.
__global__ void __launch_bounds__(kThreads) layernorm_kernel(
    const float* __restrict__ in, const float* __restrict__ scale, const float* __restrict__ bias,
    float* __restrict__ out, int64_t rows, int64_t norm, int64_t inner, float eps) {
  __shared__ double red_d[kThreads / 32];
  const int64_t len = norm * inner;
  const bool cached = len <= (int64_t)kThreads * kMaxVPT;
  const float inv_n = (float)len;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const float* x = in + row * len;
    float* y = out + row * len;
    float v[kMaxVPT];
    double s = 0.0;
    if (cached) {
#pragma unroll
      for (int k = 0; k < kMaxVPT; ++k) {
        const int64_t i = threadIdx.x + (int64_t)k * kThreads;
        v[k] = (i < len) ? x[i] : 0.0f;
        s += (double)v[k];
      }
    } else {
      for (int64_t i = threadIdx.x; i < len; i += kThreads) s += (double)x[i];
    }
    const float mean = __fdiv_rn((float)block_sum(s, red_d), inv_n);
    double q = 0.0;
    if (cached) {
#pragma unroll
      for (int k = 0; k < kMaxVPT; ++k) {
        const int64_t i = threadIdx.x + (int64_t)k * kThreads;
        if (i < len) {
          const float d = __fsub_rn(v[k], mean);
          q += (double)__fmul_rn(d, d);
        }
      }
    } else {
      for (int64_t i = threadIdx.x; i < len; i += kThreads) {
        const float d = __fsub_rn(x[i], mean);
        q += (double)__fmul_rn(d, d);
      }
    }
    const float var = __fdiv_rn((float)block_sum(q, red_d), inv_n);
    const float sd = __fsqrt_rn(__fadd_rn(var, eps));
    if (cached) {
#pragma unroll
      for (int k = 0; k < kMaxVPT; ++k) {
        const int64_t i = threadIdx.x + (int64_t)k * kThreads;
        if (i < len) {
          const int64_t a = i / inner;
          const float g = scale ? scale[a] : 1.0f;
          const float b = bias ? bias[a] : 0.0f;
          y[i] = __fadd_rn(__fmul_rn(g, __fdiv_rn(__fsub_rn(v[k], mean), sd)), b);
        }
      }
    } else {
      for (int64_t i = threadIdx.x; i < len; i += kThreads) {
        const int64_t a = i / inner;
        const float g = scale ? scale[a] : 1.0f;
        const float b = bias ? bias[a] : 0.0f;
        y[i] = __fadd_rn(__fmul_rn(g, __fdiv_rn(__fsub_rn(x[i], mean), sd)), b);
      }
    }
  }
}

// Short slabs (len <= 32 VPT): one warp per slab; `inner` == 1 indexes
// scale/bias by the element, else by i / inner (32-bit: len fits). VEC:
// 16-byte loads and stores. Statistics: pairwise fp32 sums per lane combined
// in fp64; outputs scale * ((x - mean) * (1 / sd)) + bias (within one ulp of
// the division).
// `res` (nullable): a second addend of the same shape, added to the input as
// it is loaded (one fp32 rounding, the reference's nnc_add) before the
// statistics: layernorm(in + res) in one pass (nnc_add_layernorm).
template <int VPT, bool VEC>
__global__ void __launch_bounds__(kThreads, VPT <= 8 ? 4 : 2) layernorm_warp_kernel(
    const float* __restrict__ in, const float* __restrict__ res, const float* __restrict__ scale,
    const float* __restrict__ bias, float* __restrict__ out, int64_t rows, int len, int inner,
    float eps) {
  static_assert(!VEC || VPT % 4 == 0, "vector slabs hold whole float4 runs");
  const int lane = threadIdx.x & 31;
  const int64_t step = (int64_t)gridDim.x * (kThreads / 32);
  const float inv_n = (float)len;
  // Scale and bias are the same for every slab: held in registers for short
  // slabs (VPT <= 8), re-read (L1 hits) per slab otherwise.
  constexpr bool kHold = VPT <= 8;
  float gm[kHold ? VPT : 1], bt[kHold ? VPT : 1];
  if constexpr (kHold) {
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int i = row_index<VEC>(lane, k);
      const int a = inner == 1 ? i : i / inner;
      gm[k] = (scale && i < len) ? __ldg(scale + a) : 1.0f;
      bt[k] = (bias && i < len) ? __ldg(bias + a) : 0.0f;
    }
  }
  auto load_row = [&](int64_t row, float (&v)[VPT]) {
    const float* x = in + row * len;
    const float* r = res ? res + row * len : nullptr;
    if constexpr (VEC) {
#pragma unroll
      for (int k = 0; k < VPT; k += 4) {
        const int i = row_index<true>(lane, k);
        float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
        if (i < len) t = __ldg(reinterpret_cast<const float4*>(x + i));
        if (r && i < len) {
          const float4 u = __ldg(reinterpret_cast<const float4*>(r + i));
          t = make_float4(__fadd_rn(t.x, u.x), __fadd_rn(t.y, u.y), __fadd_rn(t.z, u.z),
                          __fadd_rn(t.w, u.w));
        }
        v[k] = t.x; v[k + 1] = t.y; v[k + 2] = t.z; v[k + 3] = t.w;
      }
    } else {
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        const int i = row_index<false>(lane, k);
        v[k] = i < len ? (r ? __fadd_rn(x[i], r[i]) : x[i]) : 0.0f;
      }
    }
  };
  // Short slabs keep the next slab's loads in flight while this one reduces.
  constexpr bool kPrefetch = VPT <= 8;
  int64_t row = (int64_t)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5);
  float vn[VPT];
  if (kPrefetch && row < rows) load_row(row, vn);
  for (; row < rows; row += step) {
    float* y = out + row * len;
    float v[VPT];
    if constexpr (kPrefetch) {
#pragma unroll
      for (int k = 0; k < VPT; ++k) v[k] = vn[k];
      if (row + step < rows) load_row(row + step, vn);
    } else {
      load_row(row, v);
    }
    // Padding holds 0 and adds nothing to the sum; its squared deviations
    // are zeroed.
    const float mean = __fdiv_rn((float)warp_sum((double)tree_sum(v)), inv_n);
    float dd[VPT];
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const float d = __fsub_rn(v[k], mean);
      dd[k] = row_index<VEC>(lane, k) < len ? __fmul_rn(d, d) : 0.0f;
    }
    const float var = __fdiv_rn((float)warp_sum((double)tree_sum(dd)), inv_n);
    const float rsd = __frcp_rn(__fsqrt_rn(__fadd_rn(var, eps)));
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      float g_k, b_k;
      if constexpr (kHold) {
        g_k = gm[k];
        b_k = bt[k];
      } else {
        const int i = row_index<VEC>(lane, k);
        const int a = inner == 1 ? i : i / inner;
        g_k = (scale && i < len) ? __ldg(scale + a) : 1.0f;
        b_k = (bias && i < len) ? __ldg(bias + a) : 0.0f;
      }
      v[k] = __fadd_rn(__fmul_rn(g_k, __fmul_rn(__fsub_rn(v[k], mean), rsd)), b_k);
    }
    if constexpr (VEC) {
#pragma unroll
      for (int k = 0; k < VPT; k += 4) {
        const int i = row_index<true>(lane, k);
        if (i < len) *reinterpret_cast<float4*>(y + i) = make_float4(v[k], v[k + 1], v[k + 2], v[k + 3]);
      }
    } else {
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        const int i = row_index<false>(lane, k);
        if (i < len) y[i] = v[k];
      }
    }
  }
}

// Slabs of 513..1024 values with 16-byte rows: WPR = 4 warps per slab, 8
// values (two float4 runs) per lane, two slabs per 256-thread block in
// flight at once and the next slab's loads issued before this one reduces.
// A warp-per-slab kernel needs 32 values per lane there (128 registers, 16
// warps per SM, nothing in flight while a warp reduces: 0.60 of HBM on
// [32768, 1024]). The group's partial sums meet in shared memory in a fixed
// order (fp64), each group synchronising on its own named barrier.
template <int WPR>
__global__ void __launch_bounds__(kThreads) layernorm_group_kernel(
    const float* __restrict__ in, const float* __restrict__ res, const float* __restrict__ scale,
    const float* __restrict__ bias, float* __restrict__ out, int64_t rows, int len, int inner,
    float eps) {
  constexpr int kGroups = kThreads / 32 / WPR;
  constexpr int kRuns = 1024 / (WPR * 32 * 4);  // float4 runs per lane
  constexpr int VPT = 4 * kRuns;
  __shared__ double red[2][kGroups][WPR];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = warp / WPR, wg = warp % WPR;
  const int tg = wg * 32 + lane;  // thread within the group
  const int bar = 1 + grp;        // named barrier of the group
  const float inv_n = (float)len;
  auto idx = [&](int k) { return 4 * (tg + (k >> 2) * WPR * 32) + (k & 3); };
  auto group_sync = [&]() { asm volatile("bar.sync %0, %1;" ::"r"(bar), "r"(WPR * 32) : "memory"); };
  auto load = [&](int64_t row, float (&v)[VPT]) {
    const float* x = in + row * len;
    const float* rr = res ? res + row * len : nullptr;
#pragma unroll
    for (int r = 0; r < kRuns; ++r) {
      const int i = 4 * (tg + r * WPR * 32);
      float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
      if (i < len) t = __ldg(reinterpret_cast<const float4*>(x + i));
      if (rr && i < len) {
        const float4 u = __ldg(reinterpret_cast<const float4*>(rr + i));
        t = make_float4(__fadd_rn(t.x, u.x), __fadd_rn(t.y, u.y), __fadd_rn(t.z, u.z),
                        __fadd_rn(t.w, u.w));
      }
      v[4 * r] = t.x; v[4 * r + 1] = t.y; v[4 * r + 2] = t.z; v[4 * r + 3] = t.w;
    }
  };
  float gm[VPT], bt[VPT];
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int i = idx(k);
    const int a = inner == 1 ? i : i / inner;
    gm[k] = (scale && i < len) ? __ldg(scale + a) : 1.0f;
    bt[k] = (bias && i < len) ? __ldg(bias + a) : 0.0f;
  }
  const int64_t step = (int64_t)gridDim.x * kGroups;
  int64_t row = (int64_t)blockIdx.x * kGroups + grp;
  float vn[VPT];
  if (row < rows) load(row, vn);
  for (; row < rows; row += step) {
    float v[VPT];
#pragma unroll
    for (int k = 0; k < VPT; ++k) v[k] = vn[k];
    if (row + step < rows) load(row + step, vn);
    double part = warp_sum((double)tree_sum(v));
    if (lane == 0) red[0][grp][wg] = part;
    group_sync();
    double tot = 0.0;
#pragma unroll
    for (int w = 0; w < WPR; ++w) tot += red[0][grp][w];
    const float mean = __fdiv_rn((float)tot, inv_n);
    float dd[VPT];
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const float d = __fsub_rn(v[k], mean);
      dd[k] = idx(k) < len ? __fmul_rn(d, d) : 0.0f;
    }
    part = warp_sum((double)tree_sum(dd));
    if (lane == 0) red[1][grp][wg] = part;
    group_sync();
    double q = 0.0;
#pragma unroll
    for (int w = 0; w < WPR; ++w) q += red[1][grp][w];
    const float var = __fdiv_rn((float)q, inv_n);
    const float rsd = __frcp_rn(__fsqrt_rn(__fadd_rn(var, eps)));
    float* y = out + row * len;
#pragma unroll
    for (int r = 0; r < kRuns; ++r) {
      const int i = 4 * (tg + r * WPR * 32);
      float o[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int k = 4 * r + c;
        o[c] = __fadd_rn(__fmul_rn(gm[k], __fmul_rn(__fsub_rn(v[k], mean), rsd)), bt[k]);
      }
      if (i < len) *reinterpret_cast<float4*>(y + i) = make_float4(o[0], o[1], o[2], o[3]);
    }
    group_sync();  // the partial sums' slots are rewritten by the next slab
  }
}

// Long slabs (len <= kSmemRowMax): one 128-thread block per slab, the slab
// cached in shared memory.
__global__ void __launch_bounds__(kRowThreads) layernorm_smem_kernel(
    const float* __restrict__ in, const float* __restrict__ scale, const float* __restrict__ bias,
    float* __restrict__ out, int64_t rows, int len, int inner, float eps) {
  extern __shared__ __align__(16) float rowbuf[];
  __shared__ double red_d[4];
  const float inv_n = (float)len;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const float* x = in + row * len;
    float* y = out + row * len;
    float s = 0.0f, c = 0.0f;
    for (int i = threadIdx.x; i < len; i += kRowThreads) {
      const float t = x[i];
      rowbuf[i] = t;
      comp_add(s, c, t);
    }
    const float mean = __fdiv_rn((float)block_sum128((double)s + (double)c, red_d), inv_n);
    float q = 0.0f, qc = 0.0f;
    for (int i = threadIdx.x; i < len; i += kRowThreads) {
      const float d = __fsub_rn(rowbuf[i], mean);
      comp_add(q, qc, __fmul_rn(d, d));
    }
    __syncthreads();  // red_d is reused
    const float var = __fdiv_rn((float)block_sum128((double)q + (double)qc, red_d), inv_n);
    const float rsd = __frcp_rn(__fsqrt_rn(__fadd_rn(var, eps)));
    for (int i = threadIdx.x; i < len; i += kRowThreads) {
      const int a = inner == 1 ? i : i / inner;
      const float gm = scale ? __ldg(scale + a) : 1.0f;
      const float bt = bias ? __ldg(bias + a) : 0.0f;
      y[i] = __fadd_rn(__fmul_rn(gm, __fmul_rn(__fsub_rn(rowbuf[i], mean), rsd)), bt);
    }
    __syncthreads();  // rowbuf and red_d are reused by the next slab
  }
}

// ----------------------------------------------------------------- reduce --
// Row kernel (inner == 1): fp64 accumulation of the row, out = (float)sum
// (or (float)sum / (float)dim for the mean, ops.c:1927).
__global__ void __launch_bounds__(kThreads) reduce_row_kernel(const float* __restrict__ in,
                                                              float* __restrict__ out,
                                                              int64_t rows, int64_t dim,
                                                              int mean) {
  __shared__ double red_d[kThreads / 32];
  const bool vec = ((dim & 3) == 0) && ((((uintptr_t)in) & 15) == 0);
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    double s = 0.0;
    if (vec) {
      const float4* x4 = reinterpret_cast<const float4*>(in + row * dim);
      for (int64_t i = threadIdx.x; i < (dim >> 2); i += kThreads) {
        const float4 t = x4[i];
        s += (double)t.x + (double)t.y + (double)t.z + (double)t.w;
      }
    } else {
      const float* x = in + row * dim;
      for (int64_t i = threadIdx.x; i < dim; i += kThreads) s += (double)x[i];
    }
    s = block_sum(s, red_d);
    if (threadIdx.x == 0) {
      const float f = (float)s;
      out[row] = mean ? __fdiv_rn(f, (float)dim) : f;
    }
  }
}

// Column kernel (inner > 1): the reference's Kahan loop verbatim per column,
// so results are bit-identical to ops.c:1914-1925.
__global__ void __launch_bounds__(kThreads) reduce_col_kernel(const float* __restrict__ in,
                                                              float* __restrict__ out,
                                                              int64_t outer, int64_t dim,
                                                              int64_t inner, int mean) {
  const int64_t cols = outer * inner;
  for (int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c < cols;
       c += (int64_t)gridDim.x * blockDim.x) {
    const int64_t o = c / inner, j = c % inner;
    const float* x = in + o * dim * inner + j;
    float sum = 0.0f, comp = 0.0f;
    for (int64_t r = 0; r < dim; ++r) {
      const float yv = __fsub_rn(x[r * inner], comp);
      const float t = __fadd_rn(sum, yv);
      comp = __fsub_rn(__fsub_rn(t, sum), yv);
      sum = t;
    }
    out[o * inner + j] = mean ? __fdiv_rn(sum, (float)dim) : sum;
  }
}

bool decompose(const Tensor* t, int axis, int64_t* outer, int64_t* dim, int64_t* inner,
               const char* op) {
  int ax = axis < 0 ? axis + t->ndim : axis;
  if (ax < 0 || ax >= t->ndim) {
    fail(NNC_CUDA_ERR_INVALID, op, "axis %d out of range for ndim %d", axis, t->ndim);
    return false;
  }
  *outer = 1;
  for (int i = 0; i < ax; ++i) *outer *= t->shape[i];
  *dim = t->shape[ax];
  *inner = 1;
  for (int i = ax + 1; i < t->ndim; ++i) *inner *= t->shape[i];
  return true;
}

bool f32_plain(const Tensor* t, const char* op, const char* name) {
  if (!valid_tensor(t, op, name)) return false;
  if (elem_type(t) != NNC_DTYPE_FLOAT32 || tag_of(t) != 0) {
    fail(NNC_CUDA_ERR_UNSUPPORTED, op, "%s: needs an untagged float32 tensor", name);
    return false;
  }
  return true;
}

void reduce_impl(Tensor* in, Tensor* out, int axis, int mean, const char* op) {
  OpScope scope(op);
  if (!f32_plain(in, op, "input") || !f32_plain(out, op, "output")) return;
  trace_io(tensor_bytes(in), tensor_bytes(out));
  int64_t outer, dim, inner;
  if (!decompose(in, axis, &outer, &dim, &inner, op)) return;
  if (numel(out) != outer * inner) {
    fail(NNC_CUDA_ERR_INVALID, op, "output has %lld elements, expected %lld",
         (long long)numel(out), (long long)(outer * inner));
    return;
  }
  if (outer * inner == 0) return;
  const float* pi = (const float*)in->data;
  float* po = (float*)out->data;
  if (inner == 1) {
    const int grid = (int)(outer < (int64_t)sm_count() * 16 ? outer : (int64_t)sm_count() * 16);
    reduce_row_kernel<<<grid, kThreads, 0, ctx().stream>>>(pi, po, outer, dim, mean);
  } else {
    reduce_col_kernel<<<grid_for(outer * inner, kThreads, 8), kThreads, 0, ctx().stream>>>(
        pi, po, outer, dim, inner, mean);
  }
  check_launch(op);
}

}  // namespace
}  // namespace nnc

using namespace nnc;

extern "C" {

void nnc_softmax(Tensor* input, Tensor* output, int axis) {
  const char* op = "nnc_softmax";
  OpScope scope(op);
  if (!f32_plain(input, op, "input") || !f32_plain(output, op, "output")) return;
  trace_io(tensor_bytes(input), tensor_bytes(output));
  int64_t outer, dim, inner;
  if (!decompose(input, axis, &outer, &dim, &inner, op)) return;
  if (numel(output) < outer * dim * inner) {
    fail(NNC_CUDA_ERR_INVALID, op, "output smaller than input");
    return;
  }
  if (outer * dim * inner == 0) return;
  const float* pi = (const float*)input->data;
  float* po = (float*)output->data;
  if (inner == 1 && dim <= 1024) {
    const int64_t blocks = cdiv(outer, (int64_t)(kThreads / 32));
    const int grid = (int)(blocks < (int64_t)sm_count() * 16 ? blocks : (int64_t)sm_count() * 16);
    const int d = (int)dim;
    cudaStream_t st = ctx().stream;
    // 16-byte rows: dim % 4 == 0 and aligned bases (then every row is aligned).
    const bool vec = dim % 4 == 0 && aligned16(pi) && aligned16(po);
    if (dim <= 32)
      softmax_warp_kernel<1, false><<<grid, kThreads, 0, st>>>(pi, po, outer, d);
    else if (dim <= 64)
      softmax_warp_kernel<2, false><<<grid, kThreads, 0, st>>>(pi, po, outer, d);
    else if (dim <= 128 && vec)
      softmax_warp_kernel<4, true><<<grid, kThreads, 0, st>>>(pi, po, outer, d);
    else if (dim <= 128)
      softmax_warp_kernel<4, false><<<grid, kThreads, 0, st>>>(pi, po, outer, d);
    else if (dim <= 256 && vec)
      softmax_warp_kernel<8, true><<<grid, kThreads, 0, st>>>(pi, po, outer, d);
    else if (dim <= 256)
      softmax_warp_kernel<8, false><<<grid, kThreads, 0, st>>>(pi, po, outer, d);
    else if (dim <= 512 && vec)
      softmax_warp_kernel<16, true><<<grid, kThreads, 0, st>>>(pi, po, outer, d);
    else if (dim <= 512)
      softmax_warp_kernel<16, false><<<grid, kThreads, 0, st>>>(pi, po, outer, d);
    else if (vec)
      softmax_warp_kernel<32, true><<<grid, kThreads, 0, st>>>(pi, po, outer, d);
    else
      softmax_warp_kernel<32, false><<<grid, kThreads, 0, st>>>(pi, po, outer, d);
  } else if (inner == 1 && dim <= kSmemRowMax) {
    const size_t smem = (size_t)dim * 4;
    if (smem > 48 * 1024 &&
        !check_cuda(cudaFuncSetAttribute(softmax_smem_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)(kSmemRowMax * 4)),
                    op, "cudaFuncSetAttribute"))
      return;
    const int grid = (int)(outer < (int64_t)sm_count() * 16 ? outer : (int64_t)sm_count() * 16);
    softmax_smem_kernel<<<grid, kRowThreads, smem, ctx().stream>>>(pi, po, outer, (int)dim);
  } else if (inner == 1) {
    const int grid = (int)(outer < (int64_t)sm_count() * 8 ? outer : (int64_t)sm_count() * 8);
    softmax_row_kernel<<<grid, kThreads, 0, ctx().stream>>>(pi, po, outer, dim);
  } else {
    softmax_col_kernel<<<grid_for(outer * inner, kThreads, 8), kThreads, 0, ctx().stream>>>(
        pi, po, outer, dim, inner);
  }
  check_launch(op);
}

}  // extern "C"

namespace nnc {
namespace {
// nnc_layernorm of (input + res) when res is given (same extents as the
// input): the warp and group kernels add on load; the longer-slab kernels
// run nnc_add into the output first and normalise it in place.
void layernorm_impl(Tensor* input, Tensor* res, Tensor* scale, Tensor* bias, Tensor* output,
                    int axis, float epsilon, const char* op) {
  if (!f32_plain(input, op, "input") || !f32_plain(output, op, "output")) return;
  if (res && !f32_plain(res, op, "addend")) return;
  if ((scale && !f32_plain(scale, op, "scale")) || (bias && !f32_plain(bias, op, "bias"))) return;
  trace_io(tensor_bytes(input) + tensor_bytes(res) + tensor_bytes(scale) + tensor_bytes(bias),
           tensor_bytes(output));
  if (res && numel(res) != numel(input)) {
    fail(NNC_CUDA_ERR_INVALID, op, "the addends differ in size (%lld, %lld)",
         (long long)numel(input), (long long)numel(res));
    return;
  }
  int64_t outer, norm, inner;
  if (!decompose(input, axis, &outer, &norm, &inner, op)) return;
  if (numel(output) < outer * norm * inner) {
    fail(NNC_CUDA_ERR_INVALID, op, "output smaller than input");
    return;
  }
  if ((scale && numel(scale) < norm) || (bias && numel(bias) < norm)) {
    fail(NNC_CUDA_ERR_INVALID, op, "scale/bias shorter than the normalised axis (%lld)",
         (long long)norm);
    return;
  }
  if (outer * norm * inner == 0) return;
  const float* pi = (const float*)input->data;
  const float* pr = res ? (const float*)res->data : nullptr;
  const float* ps = scale ? (const float*)scale->data : nullptr;
  const float* pb = bias ? (const float*)bias->data : nullptr;
  float* po = (float*)output->data;
  const int64_t len = norm * inner;
  if (len <= 1024) {
    const int64_t blocks = cdiv(outer, (int64_t)(kThreads / 32));
    const int l = (int)len, in1 = (int)inner;
    cudaStream_t st = ctx().stream;
    const bool vec = len % 4 == 0 && aligned16(pi) && aligned16(po) && (!pr || aligned16(pr));
    if (len > 512 && vec) {
      const int64_t gblocks = cdiv(outer, (int64_t)(kThreads / 32 / 4));
      const int ggrid = resident_grid(layernorm_group_kernel<4>, kThreads, 0, gblocks);
      layernorm_group_kernel<4><<<ggrid, kThreads, 0, st>>>(pi, pr, ps, pb, po, outer, l, in1,
                                                          epsilon);
      check_launch(op);
      return;
    }
#define NNC_LN_WARP(VPT, VEC)                                                                  \
  layernorm_warp_kernel<VPT, VEC><<<resident_grid(layernorm_warp_kernel<VPT, VEC>, kThreads, 0, blocks), \
                                    kThreads, 0, st>>>(pi, pr, ps, pb, po, outer, l, in1, epsilon)
    if (len <= 64)
      NNC_LN_WARP(2, false);
    else if (len <= 128 && vec)
      NNC_LN_WARP(4, true);
    else if (len <= 128)
      NNC_LN_WARP(4, false);
    else if (len <= 256 && vec)
      NNC_LN_WARP(8, true);
    else if (len <= 256)
      NNC_LN_WARP(8, false);
    else if (len <= 512 && vec)
      NNC_LN_WARP(16, true);
    else if (len <= 512)
      NNC_LN_WARP(16, false);
    else if (vec)
      NNC_LN_WARP(32, true);
    else
      NNC_LN_WARP(32, false);
#undef NNC_LN_WARP
  } else if (pr) {
    // Longer slabs: the sum into the output, then the output normalised in
    // place (each kernel reads a slab before writing it).
    nnc_add(input, res, output);
    Tensor sum = *output;
    sum.ndim = input->ndim;
    sum.shape = input->shape;
    layernorm_impl(&sum, nullptr, scale, bias, output, axis, epsilon, op);
    return;
  } else if (len <= kSmemRowMax) {
    const size_t smem = (size_t)len * 4;
    if (smem > 48 * 1024 &&
        !check_cuda(cudaFuncSetAttribute(layernorm_smem_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)(kSmemRowMax * 4)),
                    op, "cudaFuncSetAttribute"))
      return;
    const int grid = (int)(outer < (int64_t)sm_count() * 16 ? outer : (int64_t)sm_count() * 16);
    layernorm_smem_kernel<<<grid, kRowThreads, smem, ctx().stream>>>(pi, ps, pb, po, outer, (int)len,
                                                                       (int)inner, epsilon);
  } else {
    const int grid = (int)(outer < (int64_t)sm_count() * 8 ? outer : (int64_t)sm_count() * 8);
    layernorm_kernel<<<grid, kThreads, 0, ctx().stream>>>(pi, ps, pb, po, outer, norm, inner, epsilon);
  }
  check_launch(op);
}
}  // namespace
}  // namespace nnc

extern "C" {

void nnc_layernorm(Tensor* input, Tensor* scale, Tensor* bias, Tensor* output, int axis,
                   float epsilon) {
  const char* op = "nnc_layernorm";
  OpScope scope(op);
  layernorm_impl(input, nullptr, scale, bias, output, axis, epsilon, op);
}

// Add -> LayerNormalization (the post-LN residual joins of a transformer at
// -O3): layernorm(a + b) with the sum never stored.
void nnc_add_layernorm(Tensor* a, Tensor* b, Tensor* scale, Tensor* bias, Tensor* output, int axis,
                       float epsilon) {
  const char* op = "nnc_add_layernorm";
  OpScope scope(op);
  if (!valid_tensor(b, op, "b")) return;
  layernorm_impl(a, b, scale, bias, output, axis, epsilon, op);
}

void nnc_reducemean(Tensor* input, Tensor* output, int axis, int keepdims) {
  (void)keepdims;  // the output layout is identical with or without the kept axis
  reduce_impl(input, output, axis, 1, "nnc_reducemean");
}

void nnc_reducesum(Tensor* input, Tensor* output, int axis, int keepdims) {
  (void)keepdims;
  reduce_impl(input, output, axis, 0, "nnc_reducesum");
}

}  // extern "C"
