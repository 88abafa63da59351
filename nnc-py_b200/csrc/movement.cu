// Data movement: reshape / flatten / squeeze / unsqueeze / identity (device
// copies), transpose, concat, split, and the NCHW <-> NHWC conversions used
// at model boundaries. All are bit-exact copies (reference ops.c:1510-1601,
// :1995-2086, :2173-2251).
#include <string.h>

#include <type_traits>

#include "common.cuh"
#include "movement.cuh"

namespace nnc {
namespace {

// out[b][c][r] = in[b][r][c] for a batch of R x C matrices: one 32 x 32
// tile per block (blockIdx.x: column tile, y: row tile, z: batch; y and z
// strided past 65535), staged in shared memory so that both the read and
// the write are coalesced; no index division. (64 x 64 tiles measured
// slower: 32.5 against 24.6 us on [256][128][256].)
constexpr int kTT = 32;
template <typename T>
__global__ void __launch_bounds__(256) batched_transpose_kernel(const T* __restrict__ in,
                                                                T* __restrict__ out, int64_t batch,
                                                                int64_t R, int64_t C,
                                                                int64_t in_bs) {
  __shared__ T tile[kTT][kTT + 1];
  const int tx = threadIdx.x % kTT, ty = threadIdx.x / kTT;  // 32 x 8 threads
  const int64_t c = (int64_t)blockIdx.x * kTT + tx;
  for (int64_t rt = blockIdx.y; rt * kTT < R; rt += gridDim.y)
  for (int64_t b = blockIdx.z; b < batch; b += gridDim.z) {
    const int64_t r0 = rt * kTT;
    const int64_t r2 = r0 + tx;
    const T* src = in + b * in_bs;
    T* dst = out + b * R * C;
#pragma unroll
    for (int j = ty; j < kTT; j += 256 / kTT) {
      const int64_t r = r0 + j;
      if (r < R && c < C) tile[j][tx] = src[r * C + c];
    }
    __syncthreads();
#pragma unroll
    for (int j = ty; j < kTT; j += 256 / kTT) {
      const int64_t c2 = (int64_t)blockIdx.x * kTT + j;
      if (r2 < R && c2 < C) dst[c2 * R + r2] = tile[tx][j];
    }
    __syncthreads();
  }
}

// The same transpose with 16-byte accesses (R and C multiples of 4, aligned
// bases): a block moves two vertically adjacent 32 x 32 tiles per step, each
// thread loading one float4 of an input row from each before either is
// stored (two 16-byte loads in flight per thread: with one, a 67 MB
// transpose ran at 0.71 of HBM), then storing one float4 of an output row
// of each; the padded tiles keep both shared-memory phases free of bank
// conflicts.
__global__ void __launch_bounds__(256) batched_transpose_vec4_kernel(const float* __restrict__ in,
                                                                     float* __restrict__ out,
                                                                     int64_t batch, int64_t R,
                                                                     int64_t C, int64_t in_bs) {
  __shared__ float tile[2][kTT][kTT + 1];
  const int q = threadIdx.x & 7, rr = threadIdx.x >> 3;  // float4 column, row within a tile
  const int64_t c0 = (int64_t)blockIdx.x * kTT;
  for (int64_t rp = blockIdx.y; 2 * rp * kTT < R; rp += gridDim.y)
  for (int64_t b = blockIdx.z; b < batch; b += gridDim.z) {
    const float* src = in + b * in_bs;
    float* dst = out + b * R * C;
    float4 v[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int64_t r = (2 * rp + h) * kTT + rr, c = c0 + 4 * q;
      v[h] = (r < R && c < C) ? __ldg(reinterpret_cast<const float4*>(src + r * C + c))
                              : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      tile[h][rr][4 * q] = v[h].x;
      tile[h][rr][4 * q + 1] = v[h].y;
      tile[h][rr][4 * q + 2] = v[h].z;
      tile[h][rr][4 * q + 3] = v[h].w;
    }
    __syncthreads();
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int64_t c = c0 + rr, r = (2 * rp + h) * kTT + 4 * q;  // output row c, columns r .. r + 3
      if (c < C && r < R)
        *reinterpret_cast<float4*>(dst + c * R + r) =
            make_float4(tile[h][4 * q][rr], tile[h][4 * q + 1][rr], tile[h][4 * q + 2][rr],
                        tile[h][4 * q + 3][rr]);
    }
    __syncthreads();
  }
}

struct Perm {
  int ndim;
  int64_t out_dims[8];
  int64_t in_strides_by_out[8];  // input stride of the dim that output dim i reads
};

// Generic N-D permutation: one thread per output element (coalesced writes).
// Idx: unsigned when every offset fits 32 bits (32-bit division is several
// times cheaper than 64-bit, and this loop is bound by its index arithmetic).
template <typename T, typename Idx>
__global__ void __launch_bounds__(256) permute_kernel(const T* __restrict__ in,
                                                      T* __restrict__ out, Idx total, Perm p) {
  for (Idx o = blockIdx.x * (Idx)blockDim.x + threadIdx.x; o < total;
       o += (Idx)gridDim.x * blockDim.x) {
    Idx rem = o, src = 0;
    for (int i = p.ndim - 1; i >= 0; --i) {
      const Idx d = (Idx)p.out_dims[i];
      const Idx q = rem / d;
      src += (rem - q * d) * (Idx)p.in_strides_by_out[i];
      rem = q;
    }
    out[o] = in[src];
  }
}

// Permutation that keeps the innermost dimension: moves rows of `inner`
// contiguous elements as V-float vectors (V = 4 or 2 by alignment).
template <int V, typename Idx>
__global__ void __launch_bounds__(256) permute_rows_kernel(const float* __restrict__ in,
                                                           float* __restrict__ out, Idx rows,
                                                           Idx inner_v, Perm p) {
  using Vec = typename std::conditional<V == 4, float4, float2>::type;
  const Idx total = rows * inner_v;
  const Idx stride = (Idx)gridDim.x * blockDim.x;
  // Four independent vectors per thread and iteration (loads in flight).
  for (Idx o0 = blockIdx.x * (Idx)blockDim.x + threadIdx.x; o0 < total; o0 += 4 * stride) {
    Vec val[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const Idx o = o0 + u * stride;
      if (o >= total) break;
      Idx rem = o / inner_v;
      const Idx v = o - rem * inner_v;
      Idx src = 0;
      for (int i = p.ndim - 2; i >= 0; --i) {
        const Idx d = (Idx)p.out_dims[i];
        const Idx q = rem / d;
        src += (rem - q * d) * (Idx)p.in_strides_by_out[i];
        rem = q;
      }
      val[u] = __ldg(reinterpret_cast<const Vec*>(in + src) + v);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const Idx o = o0 + u * stride;
      if (o >= total) break;
      reinterpret_cast<Vec*>(out)[o] = val[u];
    }
  }
}

// Device-to-device copy of n 16-byte vectors, four in flight per thread.
__global__ void __launch_bounds__(256) copy_vec4_kernel(const float4* __restrict__ in,
                                                        float4* __restrict__ out, int64_t n) {
  pdl_trigger();
  pdl_wait();
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  for (; i + 3 * stride < n; i += 4 * stride) {
    float4 v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = __ldg(in + i + j * stride);
#pragma unroll
    for (int j = 0; j < 4; ++j) out[i + j * stride] = v[j];
  }
  for (; i < n; i += stride) out[i] = __ldg(in + i);
}

bool copy_bytes(void* dst, const void* src, size_t bytes, const char* op) {
  if (bytes == 0 || dst == src) return true;
  if ((((uintptr_t)dst | (uintptr_t)src | bytes) & 15) == 0) {
    const int64_t n = (int64_t)(bytes / 16);
    launch_pdl(copy_vec4_kernel, grid_for(n, 256, 8), 256, 0, (const float4*)src, (float4*)dst, n);
    return check_launch(op);
  }
  return check_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, ctx().stream), op,
                    "cudaMemcpyAsync");
}

// Shared body of reshape / flatten / squeeze / unsqueeze: the reference
// copies numel(output) elements (ops.c:1510-1601).
void flat_copy(Tensor* input, Tensor* output, const char* op) {
  OpScope scope(op);
  if (!valid_tensor(input, op, "input") || !valid_tensor(output, op, "output")) return;
  trace_io(tensor_bytes(output), tensor_bytes(output));
  const int64_t n = numel(output);
  if (numel(input) < n) {
    fail(NNC_CUDA_ERR_INVALID, op, "input has fewer elements (%lld) than output (%lld)",
         (long long)numel(input), (long long)n);
    return;
  }
  copy_bytes(output->data, input->data, (size_t)n * elem_size(elem_type(output)), op);
}

}  // namespace

bool batched_transpose_f32(const float* in, float* out, int64_t batch, int64_t R, int64_t C,
                           const char* op, int64_t in_batch_stride) {
  if (batch * R * C == 0) return true;
  const int64_t tc = cdiv(C, kTT), tr = cdiv(R, kTT);
  if (tc > 0x7fffffff) {
    fail(NNC_CUDA_ERR_UNSUPPORTED, op, "transpose of %lld x %lld matrices", (long long)R,
         (long long)C);
    return false;
  }
  const dim3 grid((unsigned)tc, (unsigned)(tr < 65535 ? tr : 65535),
                  (unsigned)(batch < 65535 ? batch : 65535));
  const int64_t bs = in_batch_stride < 0 ? R * C : in_batch_stride;
  if (R % 4 == 0 && C % 4 == 0 && bs % 4 == 0 && aligned16(in) && aligned16(out)) {
    const int64_t tr2 = cdiv(tr, 2);  // row-tile pairs
    const dim3 grid2((unsigned)tc, (unsigned)(tr2 < 65535 ? tr2 : 65535), grid.z);
    batched_transpose_vec4_kernel<<<grid2, 256, 0, ctx().stream>>>(in, out, batch, R, C, bs);
    return check_launch(op);
  }
  batched_transpose_kernel<float><<<grid, 256, 0, ctx().stream>>>(
      in, out, batch, R, C, in_batch_stride < 0 ? R * C : in_batch_stride);
  return check_launch(op);
}

}  // namespace nnc

using namespace nnc;

extern "C" {

void nnc_reshape(Tensor* input, Tensor* output, int64_t* shape, int ndim) {
  (void)shape;
  (void)ndim;
  flat_copy(input, output, "nnc_reshape");
}
void nnc_flatten(Tensor* input, Tensor* output, int axis) {
  (void)axis;
  flat_copy(input, output, "nnc_flatten");
}
void nnc_squeeze(Tensor* input, Tensor* output, int axis) {
  (void)axis;
  flat_copy(input, output, "nnc_squeeze");
}
void nnc_unsqueeze(Tensor* input, Tensor* output, int axis) {
  (void)axis;
  flat_copy(input, output, "nnc_unsqueeze");
}

void nnc_identity(Tensor* input, Tensor* output) {
  const char* op = "nnc_identity";
  OpScope scope(op);
  if (!valid_tensor(input, op, "input") || !valid_tensor(output, op, "output")) return;
  trace_io(tensor_bytes(input), tensor_bytes(output));
  // min(numel(out), numel(in)) floats, as in ops.c:2173-2181.
  const int64_t n = numel(output) < numel(input) ? numel(output) : numel(input);
  copy_bytes(output->data, input->data, (size_t)n * sizeof(float), op);
}

}  // extern "C"

namespace nnc {
namespace {
// nnc_transpose after the scope and the NULL checks (transpose_shaped passes
// views of its tensors).
void transpose_tensors(Tensor* input, Tensor* output, int64_t* perm, int ndim, const char* op) {
  if (ndim < 1 || ndim > 8 || ndim != input->ndim || ndim != output->ndim) {
    fail(NNC_CUDA_ERR_INVALID, op, "ndim %d does not match the tensors (%d, %d)", ndim,
         input->ndim, output->ndim);
    return;
  }
  int64_t pm[8];
  for (int i = 0; i < ndim; ++i) pm[i] = perm ? perm[i] : (ndim - 1 - i);  // NULL = reverse
  for (int i = 0; i < ndim; ++i)
    if (pm[i] < 0 || pm[i] >= ndim) {
      fail(NNC_CUDA_ERR_INVALID, op, "perm[%d] = %lld out of range", i, (long long)pm[i]);
      return;
    }
  const int64_t total = numel(output);
  if (total == 0) return;
  const size_t es = elem_size(elem_type(output));
  if (es != 4 && es != 8) {
    fail(NNC_CUDA_ERR_UNSUPPORTED, op, "element size %zu not supported", es);
    return;
  }
  cudaStream_t st = ctx().stream;
  // The reference walks the output shape with the input's strides and checks
  // neither that perm is a permutation nor that the output is the permuted
  // input; such calls take the literal element-wise path.
  bool canonical = true;
  {
    bool seen[8] = {};
    for (int i = 0; i < ndim; ++i) {
      canonical &= !seen[pm[i]] && output->shape[i] == input->shape[pm[i]];
      seen[pm[i]] = true;
    }
  }
  if (!canonical) {
    int64_t in_strides[8];
    in_strides[ndim - 1] = 1;
    for (int i = ndim - 2; i >= 0; --i) in_strides[i] = in_strides[i + 1] * input->shape[i + 1];
    Perm p;
    p.ndim = ndim;
    for (int i = 0; i < ndim; ++i) {
      p.out_dims[i] = output->shape[i];
      p.in_strides_by_out[i] = in_strides[pm[i]];
    }
    const int grid = grid_for(total, 256, 8);
    if (es == 4)
      permute_kernel<float, int64_t><<<grid, 256, 0, st>>>((const float*)input->data,
                                                          (float*)output->data, total, p);
    else
      permute_kernel<int64_t, int64_t><<<grid, 256, 0, st>>>(
          (const int64_t*)input->data, (int64_t*)output->data, total, p);
    check_launch(op);
    return;
  }
  // Canonical form: drop unit dims, then merge input dims that stay adjacent
  // and in order in the output. [N,S,h,d] -> [N,h,d,S] becomes the batched
  // 2-D transpose [N][S][h*d] -> [N][h*d][S].
  int keep[8], nk = 0;  // output positions of non-unit dims
  for (int i = 0; i < ndim; ++i)
    if (output->shape[i] != 1) keep[nk++] = i;
  int64_t grp_first[8], grp_last[8];  // input dim range of each output group
  int ng = 0;
  for (int j = 0; j < nk; ++j) {
    const int64_t d = pm[keep[j]];
    // The next kept input dim after grp_last (skipping unit dims) must be d.
    bool merge = false;
    if (ng > 0) {
      int64_t nxt = grp_last[ng - 1] + 1;
      while (nxt < ndim && input->shape[nxt] == 1) ++nxt;
      merge = nxt == d;
    }
    if (merge) {
      grp_last[ng - 1] = d;
    } else {
      grp_first[ng] = d;
      grp_last[ng] = d;
      ++ng;
    }
  }
  // Groups in input order give the merged input shape; gperm maps output
  // group -> merged input dim.
  int order[8];
  for (int g = 0; g < ng; ++g) order[g] = g;
  for (int a = 1; a < ng; ++a)
    for (int b2 = a; b2 > 0 && grp_first[order[b2]] < grp_first[order[b2 - 1]]; --b2) {
      const int t = order[b2];
      order[b2] = order[b2 - 1];
      order[b2 - 1] = t;
    }
  int64_t mshape[8], mstride[8];
  int gperm[8];
  for (int k = 0; k < ng; ++k) {
    const int g = order[k];
    gperm[g] = k;
    mshape[k] = 1;
    for (int64_t d = grp_first[g]; d <= grp_last[g]; ++d) mshape[k] *= input->shape[d];
  }
  if (ng > 0) mstride[ng - 1] = 1;
  for (int k = ng - 2; k >= 0; --k) mstride[k] = mstride[k + 1] * mshape[k + 1];
  bool ident = true;
  for (int g = 0; g < ng; ++g) ident &= gperm[g] == g;
  if (ident) {  // a pure reshape: one copy
    copy_bytes(output->data, input->data, (size_t)total * es, op);
    return;
  }
  bool lead_identity = true;
  for (int g = 0; g < ng - 2; ++g) lead_identity &= (gperm[g] == g);
  if (es == 4 && ng >= 2 && lead_identity && gperm[ng - 2] == ng - 1 && gperm[ng - 1] == ng - 2) {
    const int64_t R = mshape[ng - 2], C = mshape[ng - 1];
    batched_transpose_f32((const float*)input->data, (float*)output->data, total / (R * C), R, C,
                          op);
    return;
  }
  Perm p;
  p.ndim = ng;
  for (int g = 0; g < ng; ++g) {
    p.out_dims[g] = mshape[gperm[g]];
    p.in_strides_by_out[g] = mstride[gperm[g]];
  }
  const bool small = total < (int64_t(1) << 31);
  const int64_t inner = p.out_dims[ng - 1];
  const uintptr_t align = (uintptr_t)input->data | (uintptr_t)output->data;
  if (es == 4 && gperm[ng - 1] == ng - 1 && inner % 2 == 0 && (align & 7) == 0) {
    const int V = (inner % 4 == 0 && (align & 15) == 0) ? 4 : 2;
    const int64_t rows = total / inner, iv = inner / V;
    const int grid = grid_for(total / V, 256, 8);
    const float* pi = (const float*)input->data;
    float* po = (float*)output->data;
    if (V == 4 && small)
      permute_rows_kernel<4, uint32_t><<<grid, 256, 0, st>>>(pi, po, (uint32_t)rows, (uint32_t)iv, p);
    else if (V == 4)
      permute_rows_kernel<4, int64_t><<<grid, 256, 0, st>>>(pi, po, rows, iv, p);
    else if (small)
      permute_rows_kernel<2, uint32_t><<<grid, 256, 0, st>>>(pi, po, (uint32_t)rows, (uint32_t)iv, p);
    else
      permute_rows_kernel<2, int64_t><<<grid, 256, 0, st>>>(pi, po, rows, iv, p);
  } else if (es == 4) {
    const int grid = grid_for(total, 256, 8);
    if (small)
      permute_kernel<float, uint32_t><<<grid, 256, 0, st>>>((const float*)input->data,
                                                           (float*)output->data, (uint32_t)total, p);
    else
      permute_kernel<float, int64_t><<<grid, 256, 0, st>>>((const float*)input->data,
                                                          (float*)output->data, total, p);
  } else {
    const int grid = grid_for(total, 256, 8);
    if (small)
      permute_kernel<int64_t, uint32_t><<<grid, 256, 0, st>>>(
          (const int64_t*)input->data, (int64_t*)output->data, (uint32_t)total, p);
    else
      permute_kernel<int64_t, int64_t><<<grid, 256, 0, st>>>(
          (const int64_t*)input->data, (int64_t*)output->data, total, p);
  }
  check_launch(op);
}

}  // namespace
}  // namespace nnc

extern "C" {

void nnc_transpose(Tensor* input, Tensor* output, int64_t* perm, int ndim) {
  const char* op = "nnc_transpose";
  OpScope scope(op);
  if (!valid_tensor(input, op, "input") || !valid_tensor(output, op, "output")) return;
  trace_io(tensor_bytes(input), tensor_bytes(output));
  transpose_tensors(input, output, perm, ndim, op);
}

// Reshape -> Transpose and Transpose -> Reshape as one call: the input read
// with extents in_shape (NULL: its own), permuted by perm, the output written
// as the permuted extents in row-major order whatever its own shape says
// (element counts must agree). Equals nnc_reshape / nnc_transpose /
// nnc_reshape composed: the reshapes are views, so no copy runs for them.
void nnc_transpose_shaped(Tensor* input, Tensor* output, int64_t* in_shape, int64_t* perm,
                          int ndim) {
  const char* op = "nnc_transpose_shaped";
  OpScope scope(op);
  if (!valid_tensor(input, op, "input") || !valid_tensor(output, op, "output")) return;
  trace_io(tensor_bytes(input), tensor_bytes(output));
  if (ndim < 1 || ndim > 8 || (!in_shape && ndim != input->ndim)) {
    fail(NNC_CUDA_ERR_INVALID, op, "ndim %d does not fit the input (%d)", ndim, input->ndim);
    return;
  }
  int64_t ish[8], osh[8], pm[8];
  bool seen[8] = {};
  int64_t n = 1;
  for (int i = 0; i < ndim; ++i) {
    ish[i] = in_shape ? in_shape[i] : input->shape[i];
    pm[i] = perm ? perm[i] : (ndim - 1 - i);
    if (pm[i] < 0 || pm[i] >= ndim || seen[pm[i]] || ish[i] < 0) {
      fail(NNC_CUDA_ERR_INVALID, op, "perm or shape entry %d invalid", i);
      return;
    }
    seen[pm[i]] = true;
    n *= ish[i];
  }
  if (n != numel(input) || n != numel(output)) {
    fail(NNC_CUDA_ERR_INVALID, op, "element counts differ (%lld, %lld, %lld)", (long long)n,
         (long long)numel(input), (long long)numel(output));
    return;
  }
  for (int i = 0; i < ndim; ++i) osh[i] = ish[pm[i]];
  Tensor vin = *input, vout = *output;
  vin.shape = ish;
  vin.ndim = ndim;
  vout.shape = osh;
  vout.ndim = ndim;
  transpose_tensors(&vin, &vout, pm, ndim, op);
}

void nnc_concat(Tensor** inputs, Tensor* output, int num_inputs, int axis) {
  const char* op = "nnc_concat";
  OpScope scope(op);
  if (!inputs || num_inputs < 0 || !valid_tensor(output, op, "output")) {
    fail(NNC_CUDA_ERR_INVALID, op, "invalid arguments");
    return;
  }
  trace_io(tensor_bytes(output), tensor_bytes(output));
  const int ax = axis < 0 ? axis + output->ndim : axis;
  if (ax < 0 || ax >= output->ndim) {
    fail(NNC_CUDA_ERR_INVALID, op, "axis %d out of range", axis);
    return;
  }
  // Element size follows the output dtype (int64 or 4-byte), ops.c:2011-2013.
  const size_t es = elem_type(output) == NNC_DTYPE_INT64 ? 8 : 4;
  int64_t outer = 1, inner = 1;
  for (int i = 0; i < ax; ++i) outer *= output->shape[i];
  for (int i = ax + 1; i < output->ndim; ++i) inner *= output->shape[i];
  const int64_t out_axis = output->shape[ax];
  int64_t offset = 0;
  for (int k = 0; k < num_inputs; ++k) {
    Tensor* in = inputs[k];
    if (!valid_tensor(in, op, "input") || in->ndim <= ax) {
      fail(NNC_CUDA_ERR_INVALID, op, "input %d invalid", k);
      return;
    }
    const int64_t d = in->shape[ax];
    if (offset + d > out_axis) {
      fail(NNC_CUDA_ERR_INVALID, op, "inputs exceed the output along axis %d", ax);
      return;
    }
    const size_t width = (size_t)(d * inner) * es;
    if (width && outer) {
      if (!check_cuda(cudaMemcpy2DAsync((char*)output->data + (size_t)(offset * inner) * es,
                                        (size_t)(out_axis * inner) * es, in->data, width, width,
                                        (size_t)outer, cudaMemcpyDeviceToDevice, ctx().stream),
                      op, "cudaMemcpy2DAsync"))
        return;
    }
    offset += d;
  }
}

void nnc_split(Tensor* input, Tensor** outputs, int num_outputs, int axis) {
  const char* op = "nnc_split";
  OpScope scope(op);
  if (!outputs || num_outputs <= 0 || !valid_tensor(input, op, "input")) {
    fail(NNC_CUDA_ERR_INVALID, op, "invalid arguments");
    return;
  }
  trace_io(tensor_bytes(input), tensor_bytes(input));
  const int ax = axis < 0 ? axis + input->ndim : axis;
  if (ax < 0 || ax >= input->ndim) {
    fail(NNC_CUDA_ERR_INVALID, op, "axis %d out of range", axis);
    return;
  }
  // Equal parts only (ops.c:2198-2199); dtype follows the input.
  const size_t es = elem_type(input) == NNC_DTYPE_INT64 ? 8 : 4;
  int64_t outer = 1, inner = 1;
  for (int i = 0; i < ax; ++i) outer *= input->shape[i];
  for (int i = ax + 1; i < input->ndim; ++i) inner *= input->shape[i];
  const int64_t dim = input->shape[ax];
  const int64_t part = dim / num_outputs;
  for (int k = 0; k < num_outputs; ++k) {
    if (!valid_tensor(outputs[k], op, "output")) return;
    const size_t width = (size_t)(part * inner) * es;
    if (!width || !outer) continue;
    if (!check_cuda(cudaMemcpy2DAsync(outputs[k]->data, width,
                                      (const char*)input->data + (size_t)(k * part * inner) * es,
                                      (size_t)(dim * inner) * es, width, (size_t)outer,
                                      cudaMemcpyDeviceToDevice, ctx().stream),
                    op, "cudaMemcpy2DAsync"))
      return;
  }
}

void nnc_cuda_nchw_to_nhwc(Tensor* input, Tensor* output) {
  const char* op = "nnc_cuda_nchw_to_nhwc";
  OpScope scope(op);
  if (!valid_tensor(input, op, "input") || !valid_tensor(output, op, "output")) return;
  trace_io(tensor_bytes(input), tensor_bytes(output));
  if (input->ndim != 4 || numel(output) != numel(input)) {
    fail(NNC_CUDA_ERR_INVALID, op, "expected two 4-D tensors of equal size");
    return;
  }
  const int64_t N = input->shape[0], C = input->shape[1], HW = input->shape[2] * input->shape[3];
  batched_transpose_f32((const float*)input->data, (float*)output->data, N, C, HW, op);
}

void nnc_cuda_nhwc_to_nchw(Tensor* input, Tensor* output) {
  const char* op = "nnc_cuda_nhwc_to_nchw";
  OpScope scope(op);
  if (!valid_tensor(input, op, "input") || !valid_tensor(output, op, "output")) return;
  if (input->ndim != 4 || numel(output) != numel(input)) {
    fail(NNC_CUDA_ERR_INVALID, op, "expected two 4-D tensors of equal size");
    return;
  }
  const int64_t N = input->shape[0], C = input->shape[1], HW = input->shape[2] * input->shape[3];
  batched_transpose_f32((const float*)input->data, (float*)output->data, N, HW, C, op);
}

}  // extern "C"
