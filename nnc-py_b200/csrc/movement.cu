// Data movement: reshape / flatten / squeeze / unsqueeze / identity (device
// copies), transpose, concat, split, and the NCHW <-> NHWC conversions used
// at model boundaries. All are bit-exact copies (reference ops.c:1510-1601,
// :1995-2086, :2173-2251).
#include <string.h>

#include "common.cuh"
#include "movement.cuh"

namespace nnc {
namespace {

constexpr int kTile = 32;

// out[b][c][r] = in[b][r][c] for a batch of R x C matrices (32x32 smem tiles,
// both the read and the write are coalesced).
template <typename T>
__global__ void __launch_bounds__(256) batched_transpose_kernel(const T* __restrict__ in,
                                                                T* __restrict__ out, int64_t batch,
                                                                int64_t R, int64_t C,
                                                                int64_t in_bs) {
  __shared__ T tile[kTile][kTile + 1];
  const int64_t tiles_r = cdiv(R, kTile), tiles_c = cdiv(C, kTile);
  const int64_t per_batch = tiles_r * tiles_c;
  for (int64_t t = blockIdx.x; t < batch * per_batch; t += gridDim.x) {
    const int64_t b = t / per_batch;
    const int64_t tr = (t % per_batch) / tiles_c, tc = (t % per_batch) % tiles_c;
    const T* src = in + b * in_bs;
    T* dst = out + b * R * C;
    const int64_t c = tc * kTile + threadIdx.x % kTile;
    for (int j = threadIdx.x / kTile; j < kTile; j += 256 / kTile) {
      const int64_t r = tr * kTile + j;
      if (r < R && c < C) tile[j][threadIdx.x % kTile] = src[r * C + c];
    }
    __syncthreads();
    const int64_t r2 = tr * kTile + threadIdx.x % kTile;
    for (int j = threadIdx.x / kTile; j < kTile; j += 256 / kTile) {
      const int64_t c2 = tc * kTile + j;
      if (r2 < R && c2 < C) dst[c2 * R + r2] = tile[threadIdx.x % kTile][j];
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
template <typename T>
__global__ void __launch_bounds__(256) permute_kernel(const T* __restrict__ in,
                                                      T* __restrict__ out, int64_t total,
                                                      Perm p) {
  for (int64_t o = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; o < total;
       o += (int64_t)gridDim.x * blockDim.x) {
    int64_t rem = o, src = 0;
    for (int i = p.ndim - 1; i >= 0; --i) {
      const int64_t idx = rem % p.out_dims[i];
      rem /= p.out_dims[i];
      src += idx * p.in_strides_by_out[i];
    }
    out[o] = in[src];
  }
}

// Permutation that keeps the innermost dimension: moves rows of `inner`
// contiguous elements (float4 vectors when inner % 4 == 0).
__global__ void __launch_bounds__(256) permute_rows_vec4_kernel(const float4* __restrict__ in,
                                                                float4* __restrict__ out,
                                                                int64_t rows, int64_t inner4,
                                                                Perm p) {
  const int64_t total = rows * inner4;
  for (int64_t o = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; o < total;
       o += (int64_t)gridDim.x * blockDim.x) {
    const int64_t v = o % inner4;
    int64_t rem = o / inner4, src = 0;
    for (int i = p.ndim - 2; i >= 0; --i) {
      const int64_t idx = rem % p.out_dims[i];
      rem /= p.out_dims[i];
      src += idx * p.in_strides_by_out[i];
    }
    out[o] = in[src / 4 + v];
  }
}

bool copy_bytes(void* dst, const void* src, size_t bytes, const char* op) {
  if (bytes == 0 || dst == src) return true;
  return check_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, ctx().stream), op,
                    "cudaMemcpyAsync");
}

// Shared body of reshape / flatten / squeeze / unsqueeze: the reference
// copies numel(output) elements (ops.c:1510-1601).
void flat_copy(Tensor* input, Tensor* output, const char* op) {
  OpScope scope(op);
  if (!valid_tensor(input, op, "input") || !valid_tensor(output, op, "output")) return;
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
  const int64_t tiles = batch * cdiv(R, kTile) * cdiv(C, kTile);
  const int grid = (int)(tiles < (int64_t)sm_count() * 16 ? tiles : (int64_t)sm_count() * 16);
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
  // min(numel(out), numel(in)) floats, as in ops.c:2173-2181.
  const int64_t n = numel(output) < numel(input) ? numel(output) : numel(input);
  copy_bytes(output->data, input->data, (size_t)n * sizeof(float), op);
}

void nnc_transpose(Tensor* input, Tensor* output, int64_t* perm, int ndim) {
  const char* op = "nnc_transpose";
  OpScope scope(op);
  if (!valid_tensor(input, op, "input") || !valid_tensor(output, op, "output")) return;
  if (ndim < 1 || ndim > 8 || ndim != input->ndim || ndim != output->ndim) {
    fail(NNC_CUDA_ERR_INVALID, op, "ndim %d does not match the tensors (%d, %d)", ndim,
         input->ndim, output->ndim);
    return;
  }
  int64_t pm[8];
  for (int i = 0; i < ndim; ++i) pm[i] = perm ? perm[i] : (ndim - 1 - i);  // NULL = reverse
  int64_t in_strides[8];
  in_strides[ndim - 1] = 1;
  for (int i = ndim - 2; i >= 0; --i) in_strides[i] = in_strides[i + 1] * input->shape[i + 1];
  Perm p;
  p.ndim = ndim;
  for (int i = 0; i < ndim; ++i) {
    if (pm[i] < 0 || pm[i] >= ndim) {
      fail(NNC_CUDA_ERR_INVALID, op, "perm[%d] = %lld out of range", i, (long long)pm[i]);
      return;
    }
    p.out_dims[i] = output->shape[i];
    p.in_strides_by_out[i] = in_strides[pm[i]];
  }
  const int64_t total = numel(output);
  if (total == 0) return;
  const size_t es = elem_size(elem_type(output));
  if (es != 4 && es != 8) {
    fail(NNC_CUDA_ERR_UNSUPPORTED, op, "element size %zu not supported", es);
    return;
  }
  // Batched 2-D transpose of the last two dims (leading dims in order).
  bool lead_identity = true;
  for (int i = 0; i < ndim - 2; ++i) lead_identity &= (pm[i] == i);
  if (es == 4 && ndim >= 2 && lead_identity && pm[ndim - 2] == ndim - 1 &&
      pm[ndim - 1] == ndim - 2) {
    const int64_t R = input->shape[ndim - 2], C = input->shape[ndim - 1];
    batched_transpose_f32((const float*)input->data, (float*)output->data, total / (R * C), R, C,
                          op);
    return;
  }
  const int64_t inner = output->shape[ndim - 1];
  if (es == 4 && pm[ndim - 1] == ndim - 1 && inner % 4 == 0 && aligned16(input->data) &&
      aligned16(output->data)) {
    permute_rows_vec4_kernel<<<grid_for(total / 4, 256, 8), 256, 0, ctx().stream>>>(
        (const float4*)input->data, (float4*)output->data, total / inner, inner / 4, p);
  } else if (es == 4) {
    permute_kernel<float><<<grid_for(total, 256, 8), 256, 0, ctx().stream>>>(
        (const float*)input->data, (float*)output->data, total, p);
  } else {
    permute_kernel<int64_t><<<grid_for(total, 256, 8), 256, 0, ctx().stream>>>(
        (const int64_t*)input->data, (int64_t*)output->data, total, p);
  }
  check_launch(op);
}

void nnc_concat(Tensor** inputs, Tensor* output, int num_inputs, int axis) {
  const char* op = "nnc_concat";
  OpScope scope(op);
  if (!inputs || num_inputs < 0 || !valid_tensor(output, op, "output")) {
    fail(NNC_CUDA_ERR_INVALID, op, "invalid arguments");
    return;
  }
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
