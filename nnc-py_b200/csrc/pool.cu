// 2-D max / average pooling (reference ops.c:316-461).
//
// Window semantics are the reference's: the window [o*stride - pad,
// o*stride - pad + k) is clamped to the input, so padding never contributes;
// only the top/left pad is passed and the output extent comes from
// output->shape. Max keeps the first in-window value and replaces it only by
// a strictly greater one; an empty window yields -3.402823e38f. Average sums
// in row-major window order in fp32 and divides by the in-bounds count
// (0 for an empty window). Both are bit-identical to the reference.
//
// Layouts: NCHW (untagged tensors) — one thread per output element, writes
// coalesced along W; NHWC (NNC_CUDA_TAG_NHWC) — one thread per output pixel
// and 4-channel group, 128-bit loads/stores along C.
#include "common.cuh"

namespace nnc {
namespace {

constexpr float kEmptyMax = -3.402823e38f;

struct PoolGeom {
  int N, C, H, W, OH, OW, kh, kw, sh, sw, ph, pw;
};

__device__ __forceinline__ void window(const PoolGeom& g, int oh, int ow, int& h0, int& h1,
                                       int& w0, int& w1) {
  h0 = oh * g.sh - g.ph;
  w0 = ow * g.sw - g.pw;
  h1 = h0 + g.kh;
  w1 = w0 + g.kw;
  h0 = h0 < 0 ? 0 : h0;
  w0 = w0 < 0 ? 0 : w0;
  h1 = h1 > g.H ? g.H : h1;
  w1 = w1 > g.W ? g.W : w1;
}

// FULL2: 2x2 windows, stride 2, no padding, every window inside the input and
// W even — the two values of a window row are one aligned 8-byte load.
template <bool MAX, typename Idx, bool FULL2>
__global__ void __launch_bounds__(256) pool_nchw_kernel(const float* __restrict__ in,
                                                        float* __restrict__ out, PoolGeom g) {
  const Idx total = (Idx)g.N * g.C * g.OH * g.OW;
  for (Idx idx = blockIdx.x * (Idx)blockDim.x + threadIdx.x; idx < total;
       idx += (Idx)gridDim.x * blockDim.x) {
    const Idx r = idx / g.OW;
    const int ow = (int)(idx - r * g.OW);
    const Idx nc = r / g.OH;
    const int oh = (int)(r - nc * g.OH);
    const float* plane = in + nc * g.H * g.W;
    if constexpr (FULL2) {
      const float2 t0 = __ldg(reinterpret_cast<const float2*>(plane + (2 * oh) * g.W + 2 * ow));
      const float2 t1 =
          __ldg(reinterpret_cast<const float2*>(plane + (2 * oh + 1) * g.W + 2 * ow));
      if (MAX) {
        float m = t0.x;
        if (t0.y > m) m = t0.y;
        if (t1.x > m) m = t1.x;
        if (t1.y > m) m = t1.y;
        out[idx] = m;
      } else {
        const float s = __fadd_rn(__fadd_rn(__fadd_rn(t0.x, t0.y), t1.x), t1.y);
        out[idx] = __fdiv_rn(s, 4.0f);
      }
      continue;
    }
    int h0, h1, w0, w1;
    window(g, oh, ow, h0, h1, w0, w1);
    if (MAX) {
      float m = kEmptyMax;
      bool has = false;
      for (int h = h0; h < h1; ++h)
        for (int w = w0; w < w1; ++w) {
          const float v = plane[h * g.W + w];
          if (!has || v > m) {
            m = v;
            has = true;
          }
        }
      out[idx] = m;
    } else {
      float s = 0.0f;
      int cnt = 0;
      for (int h = h0; h < h1; ++h)
        for (int w = w0; w < w1; ++w) {
          s = __fadd_rn(s, plane[h * g.W + w]);
          ++cnt;
        }
      out[idx] = cnt > 0 ? __fdiv_rn(s, (float)cnt) : 0.0f;
    }
  }
}

// Idx: the index type, int when every input and output element offset fits
// (32-bit division and multiplication are several times cheaper than 64-bit,
// and this loop is bound by its index arithmetic otherwise).
template <bool MAX, int V, typename Idx>
__global__ void __launch_bounds__(256) pool_nhwc_kernel(const float* __restrict__ in,
                                                        float* __restrict__ out, PoolGeom g) {
  pdl_trigger();
  pdl_wait();
  // V channels per thread (4 or 2 with 16- or 8-byte alignment, else 1).
  const Idx cg = g.C / V;
  const Idx total = (Idx)g.N * g.OH * g.OW * cg;
  for (Idx idx = blockIdx.x * (Idx)blockDim.x + threadIdx.x; idx < total;
       idx += (Idx)gridDim.x * blockDim.x) {
    const int c = (int)(idx % cg) * V;
    const Idx p = idx / cg;
    const int ow = (int)(p % g.OW);
    const Idx q = p / g.OW;
    const int oh = (int)(q % g.OH);
    const int n = (int)(q / g.OH);
    int h0, h1, w0, w1;
    window(g, oh, ow, h0, h1, w0, w1);
    const float* img = in + (Idx)n * g.H * g.W * g.C + c;
    float acc[V];
    bool has = false;
    int cnt = 0;
#pragma unroll
    for (int j = 0; j < V; ++j) acc[j] = MAX ? kEmptyMax : 0.0f;
    for (int h = h0; h < h1; ++h)
      for (int w = w0; w < w1; ++w) {
        const float* src = img + ((Idx)h * g.W + w) * g.C;
        float v[V];
        if constexpr (V == 4) {
          const float4 t = *reinterpret_cast<const float4*>(src);
          v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
        } else if constexpr (V == 2) {
          const float2 t = *reinterpret_cast<const float2*>(src);
          v[0] = t.x; v[1] = t.y;
        } else {
          v[0] = src[0];
        }
#pragma unroll
        for (int j = 0; j < V; ++j) {
          if (MAX) {
            if (!has || v[j] > acc[j]) acc[j] = v[j];
          } else {
            acc[j] = __fadd_rn(acc[j], v[j]);
          }
        }
        has = true;
        ++cnt;
      }
    float* dst = out + p * g.C + c;
#pragma unroll
    for (int j = 0; j < V; ++j) {
      if (!MAX) acc[j] = cnt > 0 ? __fdiv_rn(acc[j], (float)cnt) : 0.0f;
    }
    if constexpr (V == 4) {
      *reinterpret_cast<float4*>(dst) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    } else if constexpr (V == 2) {
      *reinterpret_cast<float2*>(dst) = make_float2(acc[0], acc[1]);
    } else {
      dst[0] = acc[0];
    }
  }
}

// Channels-last with few channels (C even, at most 8; LeNet's 6): one thread
// per output pixel takes all its channels as float2 pairs, so the index
// arithmetic is paid once per pixel instead of once per pair. Same window
// order and tie rules as pool_nhwc_kernel.
template <bool MAX>
__global__ void __launch_bounds__(256) pool_nhwc_pixel_kernel(const float* __restrict__ in,
                                                              float* __restrict__ out, PoolGeom g) {
  const int pairs = g.C / 2;
  const int total = g.N * g.OH * g.OW;  // host: fits 32 bits
  for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < total; p += gridDim.x * blockDim.x) {
    const int ow = p % g.OW;
    const int q = p / g.OW;
    const int oh = q % g.OH;
    const int n = q / g.OH;
    int h0, h1, w0, w1;
    window(g, oh, ow, h0, h1, w0, w1);
    const float* img = in + (int64_t)n * g.H * g.W * g.C;
    float2 acc[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[j] = MAX ? make_float2(kEmptyMax, kEmptyMax) : make_float2(0.f, 0.f);
    bool has = false;
    int cnt = 0;
    for (int h = h0; h < h1; ++h)
      for (int w = w0; w < w1; ++w) {
        const float2* src = reinterpret_cast<const float2*>(img + (h * g.W + w) * g.C);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (j >= pairs) break;
          const float2 v = __ldg(src + j);
          if (MAX) {
            if (!has || v.x > acc[j].x) acc[j].x = v.x;
            if (!has || v.y > acc[j].y) acc[j].y = v.y;
          } else {
            acc[j].x = __fadd_rn(acc[j].x, v.x);
            acc[j].y = __fadd_rn(acc[j].y, v.y);
          }
        }
        has = true;
        ++cnt;
      }
    float2* dst = reinterpret_cast<float2*>(out + (int64_t)p * g.C);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (j >= pairs) break;
      float2 o = acc[j];
      if (!MAX) {
        o.x = cnt > 0 ? __fdiv_rn(o.x, (float)cnt) : 0.0f;
        o.y = cnt > 0 ? __fdiv_rn(o.y, (float)cnt) : 0.0f;
      }
      dst[j] = o;
    }
  }
}

template <bool MAX>
void launch_pool(const float* pi, float* po, const PoolGeom& g, bool nhwc) {
  const int64_t total = (int64_t)g.N * g.C * g.OH * g.OW;
  // 32-bit indexing when every offset (and the grid-stride overshoot) fits.
  const int64_t in_elems = (int64_t)g.N * g.C * g.H * g.W;
  const bool small = in_elems < (int64_t(1) << 30) && total < (int64_t(1) << 30);
  cudaStream_t st = ctx().stream;
  if (!nhwc) {
    const int grid = grid_for(total, 256, 8);
    const bool full2 = g.kh == 2 && g.kw == 2 && g.sh == 2 && g.sw == 2 && g.ph == 0 &&
                       g.pw == 0 && g.W % 2 == 0 && 2 * g.OH <= g.H && 2 * g.OW <= g.W &&
                       ((uintptr_t)pi & 7) == 0;
    if (small && full2)
      pool_nchw_kernel<MAX, int, true><<<grid, 256, 0, st>>>(pi, po, g);
    else if (small)
      pool_nchw_kernel<MAX, int, false><<<grid, 256, 0, st>>>(pi, po, g);
    else if (full2)
      pool_nchw_kernel<MAX, int64_t, true><<<grid, 256, 0, st>>>(pi, po, g);
    else
      pool_nchw_kernel<MAX, int64_t, false><<<grid, 256, 0, st>>>(pi, po, g);
  } else if (g.C % 4 == 0 && aligned16(pi) && aligned16(po) &&
             total / 4 >= (int64_t)2 * sm_count() * 256) {
    // Four channels per thread; with fewer outputs (a global pool over a
    // small batch) one channel per thread instead, four times the threads.
    const int grid = grid_for(total / 4, 256, 8);
    if (small)
      launch_pdl(pool_nhwc_kernel<MAX, 4, int>, grid, 256, 0, pi, po, g);
    else
      launch_pdl(pool_nhwc_kernel<MAX, 4, int64_t>, grid, 256, 0, pi, po, g);
  } else if (g.C % 2 == 0 && g.C <= 8 && small && (((uintptr_t)pi | (uintptr_t)po) & 7) == 0) {
    pool_nhwc_pixel_kernel<MAX><<<grid_for(total / g.C, 256, 8), 256, 0, st>>>(pi, po, g);
  } else if (g.C % 2 == 0 && (((uintptr_t)pi | (uintptr_t)po) & 7) == 0) {
    const int grid = grid_for(total / 2, 256, 8);
    if (small)
      launch_pdl(pool_nhwc_kernel<MAX, 2, int>, grid, 256, 0, pi, po, g);
    else
      launch_pdl(pool_nhwc_kernel<MAX, 2, int64_t>, grid, 256, 0, pi, po, g);
  } else {
    const int grid = grid_for(total, 256, 8);
    if (small)
      launch_pdl(pool_nhwc_kernel<MAX, 1, int>, grid, 256, 0, pi, po, g);
    else
      launch_pdl(pool_nhwc_kernel<MAX, 1, int64_t>, grid, 256, 0, pi, po, g);
  }
}

template <bool MAX>
void pool_impl(Tensor* input, Tensor* output, int kh, int kw, int sh, int sw, int ph, int pw,
               const char* op) {
  OpScope scope(op);
  if (!valid_tensor(input, op, "input") || !valid_tensor(output, op, "output")) return;
  trace_io(tensor_bytes(input), tensor_bytes(output));
  if (input->ndim != 4 || output->ndim != 4) {
    // The reference returns silently for non-4-D tensors (ops.c:332-334).
    fail(NNC_CUDA_ERR_INVALID, op, "expected 4-D tensors");
    return;
  }
  if (elem_type(input) != NNC_DTYPE_FLOAT32 || elem_type(output) != NNC_DTYPE_FLOAT32) {
    fail(NNC_CUDA_ERR_UNSUPPORTED, op, "only float32 is supported");
    return;
  }
  if (is_nhwc(input) != is_nhwc(output)) {
    fail(NNC_CUDA_ERR_UNSUPPORTED, op, "input and output layouts differ");
    return;
  }
  if (kh <= 0 || kw <= 0 || sh <= 0 || sw <= 0) {
    fail(NNC_CUDA_ERR_INVALID, op, "kernel and stride must be positive");
    return;
  }
  PoolGeom g{(int)input->shape[0],  (int)input->shape[1],  (int)input->shape[2],
             (int)input->shape[3],  (int)output->shape[2], (int)output->shape[3],
             kh, kw, sh, sw, ph, pw};
  if (output->shape[0] != g.N || output->shape[1] != g.C) {
    fail(NNC_CUDA_ERR_INVALID, op, "output N/C differ from the input");
    return;
  }
  const int64_t total = (int64_t)g.N * g.C * g.OH * g.OW;
  if (total == 0) return;
  launch_pool<MAX>((const float*)input->data, (float*)output->data, g, is_nhwc(input));
  check_launch(op);
}

}  // namespace

// Max pooling of a float32 tensor already on the device (for fused callers
// whose pooled input is an intermediate): the same kernels and semantics as
// nnc_maxpool2d. Returns false with the status set on a launch failure.
bool launch_maxpool_f32(const float* in, float* out, int N, int C, int H, int W, int OH, int OW,
                        int kh, int kw, int sh, int sw, int ph, int pw, bool nhwc, const char* op) {
  PoolGeom g{N, C, H, W, OH, OW, kh, kw, sh, sw, ph, pw};
  if ((int64_t)N * C * OH * OW == 0) return true;
  launch_pool<true>(in, out, g, nhwc);
  return check_launch(op);
}

// Average pooling between two device buffers (nnc_avgpool2d semantics), for
// fused callers whose pooled output is an intermediate.
bool launch_avgpool_f32(const float* in, float* out, int N, int C, int H, int W, int OH, int OW,
                        int kh, int kw, int sh, int sw, int ph, int pw, bool nhwc, const char* op) {
  PoolGeom g{N, C, H, W, OH, OW, kh, kw, sh, sw, ph, pw};
  if ((int64_t)N * C * OH * OW == 0) return true;
  launch_pool<false>(in, out, g, nhwc);
  return check_launch(op);
}

}  // namespace nnc

extern "C" {

void nnc_maxpool2d(Tensor* input, Tensor* output, int kernel_h, int kernel_w, int stride_h,
                   int stride_w, int pad_h, int pad_w) {
  nnc::pool_impl<true>(input, output, kernel_h, kernel_w, stride_h, stride_w, pad_h, pad_w,
                       "nnc_maxpool2d");
}

void nnc_avgpool2d(Tensor* input, Tensor* output, int kernel_h, int kernel_w, int stride_h,
                   int stride_w, int pad_h, int pad_w) {
  nnc::pool_impl<false>(input, output, kernel_h, kernel_w, stride_h, stride_w, pad_h, pad_w,
                        "nnc_avgpool2d");
}

}  // extern "C"
