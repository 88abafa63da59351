// The rest of the reference's operator library (runtime/x86/ops.c:2088-3116):
// cast, comparisons and logic, shape / constant-of-shape / expand / tile,
// gather, batch normalisation (an empty TODO in the reference) and LSTM.
// None of them is on a BASELINE model's path; they make every operator a
// generated model.c can call available on the GPU, with the reference's
// semantics including its quirks (each kernel cites the lines it follows).
//
// HBM-bound grid-stride kernels; LSTM is one CTA stepping through the
// reference's sequential recurrence. Built with -fmad=false: the LSTM cell's
// f * c + i * g is two roundings, as in the reference's C.
#include <math.h>
#include <stdint.h>

#include <algorithm>

#include "common.cuh"

namespace nnc {
namespace {

constexpr int kThreads = 256;

// --------------------------------------------------------------- cast ----
// x86 float -> integer conversion (cvttss2si): truncation toward zero, and
// the "integer indefinite" value (the type's minimum) for NaN and for values
// outside the type's range, where CUDA's conversions would saturate.
__device__ __forceinline__ int32_t f2i32_x86(float x) {
  if (!(x > -2147483904.0f && x < 2147483648.0f)) return INT32_MIN;
  return (int32_t)x;
}
__device__ __forceinline__ int64_t f2i64_x86(float x) {
  if (!(x >= -9223372036854775808.0f && x < 9223372036854775808.0f)) return INT64_MIN;
  return (int64_t)x;
}

// to: 0 float32 (from bool), 2 int32, 6 int64, 5 bool; src_bool: input is uint8.
__global__ void cast_kernel(const void* __restrict__ in, void* __restrict__ out, int64_t n, int to,
                            int src_bool) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float f = src_bool ? 0.0f : static_cast<const float*>(in)[i];
    const uint8_t u = src_bool ? static_cast<const uint8_t*>(in)[i] : 0;
    switch (to) {
      case NNC_DTYPE_FLOAT32: static_cast<float*>(out)[i] = (float)u; break;
      case NNC_DTYPE_INT32:
        static_cast<int32_t*>(out)[i] = src_bool ? (int32_t)u : f2i32_x86(f);
        break;
      case NNC_DTYPE_INT64:
        static_cast<int64_t*>(out)[i] = src_bool ? (int64_t)u : f2i64_x86(f);
        break;
      default: static_cast<uint8_t*>(out)[i] = f != 0.0f ? 1 : 0; break;  // bool from float
    }
  }
}

// ------------------------------------------------- binary compare / logic --
enum CmpOp : int { kEqual = 0, kAnd = 1 };

// nnc_equal / nnc_and (ops.c:2342-2432): float inputs, float 1/0 output. The
// reference compares index by index over min(n, a_n, b_n), then broadcasts
// the shorter operand (one element, or a suffix of n' < n elements, taken
// modulo n') over the rest when the other has n elements; with both shorter
// than n the tail is left untouched. Index by index equals the modular
// broadcast on the first part, so one formula covers the written range.
template <int OP>
__global__ void cmp_kernel(const float* __restrict__ a, const float* __restrict__ b,
                           float* __restrict__ out, int64_t n, int64_t an, int64_t bn) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float x = a[i < an ? i : i % an], y = b[i < bn ? i : i % bn];
    bool r;
    if constexpr (OP == kEqual) r = x == y;
    else r = x != 0.0f && y != 0.0f;
    out[i] = r ? 1.0f : 0.0f;
  }
}

// nnc_greater (ops.c:2655-2672): out[i] = a[i % a_n] > b[i % b_n] as a bool byte.
__global__ void greater_kernel(const float* __restrict__ a, const float* __restrict__ b,
                               uint8_t* __restrict__ out, int64_t n, int64_t an, int64_t bn) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = a[i % an] > b[i % bn] ? 1 : 0;
}

// nnc_or / nnc_not (ops.c:2674-2703): bool bytes, n = numel(output), no broadcast.
__global__ void or_kernel(const uint8_t* __restrict__ a, const uint8_t* __restrict__ b,
                          uint8_t* __restrict__ out, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = (a[i] || b[i]) ? 1 : 0;
}
__global__ void not_kernel(const uint8_t* __restrict__ in, uint8_t* __restrict__ out, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = in[i] ? 0 : 1;
}

// ------------------------------------------------------ fills and copies --
__global__ void fill_kernel(float* __restrict__ out, int64_t n, float v) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = v;
}

struct Dims8 {
  int64_t v[8];
};
__global__ void write_i64_kernel(int64_t* __restrict__ out, Dims8 vals, int n) {
  if (threadIdx.x < n) out[threadIdx.x] = vals.v[threadIdx.x];
}

// out[i] = in[i % in_n] for ELEM-byte elements (expand, gather's fallback).
template <typename T>
__global__ void modular_copy_kernel(const T* __restrict__ in, T* __restrict__ out, int64_t n,
                                    int64_t in_n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = in[i % in_n];
}

// nnc_tile (ops.c:2264-2336): the output index is decomposed over the
// output's extents and coordinate d (d < input rank) maps to coord %
// in_shape[d] at the input's row-major stride; the repeats only shape the
// output (they never enter the index map).
struct TileGeom {
  int out_ndim, in_ndim;
  int64_t out_shape[8], in_shape[8], in_stride[8];
};
__global__ void tile_kernel(const float* __restrict__ in, float* __restrict__ out, int64_t n,
                            TileGeom g) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t coords[8];
    int64_t t = i;
    for (int d = g.out_ndim - 1; d >= 0; --d) {
      coords[d] = t % g.out_shape[d];
      t /= g.out_shape[d];
    }
    int64_t src = 0;
    for (int d = 0; d < g.in_ndim; ++d) src += (coords[d] % g.in_shape[d]) * g.in_stride[d];
    out[i] = in[src];
  }
}

// --------------------------------------------------------------- gather --
// nnc_gather (ops.c:2705-2900) is a cascade of special cases; the host picks
// the case the reference would take and this kernel applies its index map.
// The index is read, normalised (negative + extent) and clamped on the device.
enum GatherCase : int {
  kG_I64Rank1Scalar,  // out[0] = data[g] (int64)
  kG_I64Rows,         // out[i] = data[g * copy + i], i < copy (int64)
  kG_F32Rank1Scalar,  // out[i] = data[g] for every output element
  kG_F32Rank2Scalar,  // out[i][j] = axis 0 ? data[g][j] : data[i][g]
  kG_F32Rank3Axis0Out2,
  kG_F32Rank3Axis0Out3,
  kG_F32Rank3Axis1,
  kG_F32Rank3Axis2,
  kG_I64Rank1List,    // out[k] = data[idx[k]] (int64)
  kG_F32Rank2List,    // axis 0: rows idx[k]; axis 1: columns idx[k]
};
struct GatherArgs {
  int kase, axis;
  int64_t out_n, num_idx;
  int64_t d0, d1, d2;   // data extents (1 past the rank)
  int64_t o0, o1, o2;   // output extents
  int64_t axis_extent;  // data->shape[axis]
  int64_t copy;         // kG_I64Rows: elements after the axis
};
__device__ __forceinline__ int64_t clamp_index(int64_t g, int64_t extent) {
  if (g < 0) g += extent;
  if (g < 0) g = 0;
  if (g >= extent) g = extent - 1;
  return g;
}
__global__ void gather_kernel(const void* __restrict__ data, const int64_t* __restrict__ idx,
                              void* __restrict__ out, GatherArgs a) {
  const float* df = static_cast<const float*>(data);
  const int64_t* dl = static_cast<const int64_t*>(data);
  float* of = static_cast<float*>(out);
  int64_t* ol = static_cast<int64_t*>(out);
  const int64_t g = clamp_index(idx[0], a.axis_extent);
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  const int64_t start = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  switch (a.kase) {
    case kG_I64Rank1Scalar:
      if (start == 0) ol[0] = dl[g];
      break;
    case kG_I64Rows:
      for (int64_t i = start; i < a.copy; i += step) ol[i] = dl[g * a.copy + i];
      break;
    case kG_F32Rank1Scalar:
      for (int64_t i = start; i < a.out_n; i += step) of[i] = df[g];
      break;
    case kG_F32Rank2Scalar:
      for (int64_t e = start; e < a.o0 * a.o1; e += step) {
        const int64_t i = e / a.o1, j = e % a.o1;
        of[e] = a.axis == 0 ? df[g * a.d1 + j] : df[i * a.d1 + g];
      }
      break;
    case kG_F32Rank3Axis0Out2:
      for (int64_t e = start; e < a.d1 * a.d2; e += step) of[e] = df[g * a.d1 * a.d2 + e];
      break;
    case kG_F32Rank3Axis0Out3:
      for (int64_t e = start; e < a.o0 * a.o1 * a.o2; e += step) {
        const int64_t jk = e % (a.o1 * a.o2), j = jk / a.o2, k = jk % a.o2;
        of[e] = df[g * a.d1 * a.d2 + j * a.d2 + k];
      }
      break;
    case kG_F32Rank3Axis1:
      for (int64_t e = start; e < a.d0 * a.d2; e += step) {
        const int64_t i = e / a.d2, k = e % a.d2;
        of[e] = df[i * a.d1 * a.d2 + g * a.d2 + k];
      }
      break;
    case kG_F32Rank3Axis2:
      for (int64_t e = start; e < a.d0 * a.d1; e += step) {
        const int64_t i = e / a.d1, j = e % a.d1;
        of[e] = df[i * a.d1 * a.d2 + j * a.d2 + g];
      }
      break;
    case kG_I64Rank1List:
      for (int64_t k = start; k < a.num_idx; k += step) ol[k] = dl[clamp_index(idx[k], a.d0)];
      break;
    case kG_F32Rank2List:
      if (a.axis == 0) {
        for (int64_t e = start; e < a.num_idx * a.d1; e += step) {
          const int64_t k = e / a.d1, j = e % a.d1;
          of[k * a.d1 + j] = df[clamp_index(idx[k], a.axis_extent) * a.d1 + j];
        }
      } else {
        for (int64_t e = start; e < a.num_idx * a.d0; e += step) {
          const int64_t k = e / a.d0, i = e % a.d0;
          of[i * a.num_idx + k] = df[i * a.d1 + clamp_index(idx[k], a.axis_extent)];
        }
      }
      break;
  }
}

// ----------------------------------------------------------------- LSTM --
// nnc_lstm (ops.c:2928-3116) in the reference's order: directions, then time
// steps, then batch items, ONE hidden/cell state carried through all of them
// (the reference does not keep a state per batch item). Thread r computes
// row r of the four gates with the reference's sequential fp32 sums
// (W x first, then R h, then the two biases added together), so the sums are
// bit-identical; sigmoid = 1 / (1 + expf(-x)) and tanhf are CUDA's.
__global__ void lstm_kernel(const float* __restrict__ X, const float* __restrict__ W,
                            const float* __restrict__ R, const float* __restrict__ Bv,
                            float* __restrict__ Y, float* __restrict__ Yh, float* __restrict__ Yc,
                            int T, int Bn, int I, int H, int dirs) {
  extern __shared__ float st[];  // h, c, h_next, c_next
  float* h = st;
  float* c = st + H;
  float* hn = st + 2 * H;
  float* cn = st + 3 * H;
  for (int dir = 0; dir < dirs; ++dir) {
    for (int r = threadIdx.x; r < H; r += blockDim.x) h[r] = c[r] = 0.0f;
    __syncthreads();
    const float* Wd = W + (int64_t)dir * 4 * H * I;
    const float* Rd = R + (int64_t)dir * 4 * H * H;
    const float* Bd = Bv ? Bv + (int64_t)dir * 8 * H : nullptr;
    for (int t = 0; t < T; ++t) {
      const int tt = dir == 1 ? T - 1 - t : t;
      for (int b = 0; b < Bn; ++b) {
        const float* x = X + ((int64_t)tt * Bn + b) * I;
        for (int r = threadIdx.x; r < H; r += blockDim.x) {
          float gate[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {  // I, O, F, C
            const float* wr = Wd + ((int64_t)q * H + r) * I;
            const float* rr = Rd + ((int64_t)q * H + r) * H;
            float s = 0.0f;
            for (int j = 0; j < I; ++j) s = s + wr[j] * x[j];
            for (int j = 0; j < H; ++j) s = s + rr[j] * h[j];
            if (Bd) s = s + (Bd[q * H + r] + Bd[(4 + q) * H + r]);
            gate[q] = s;
          }
          const float ig = 1.0f / (1.0f + expf(-gate[0]));
          const float og = 1.0f / (1.0f + expf(-gate[1]));
          const float fg = 1.0f / (1.0f + expf(-gate[2]));
          const float gg = tanhf(gate[3]);
          const float cv = fg * c[r] + ig * gg;
          cn[r] = cv;
          hn[r] = og * tanhf(cv);
        }
        __syncthreads();
        // Y[t][dir][b][:] — the reference indexes Y by t, not by the
        // reversed step, for the backward direction too.
        float* y = Y + (((int64_t)t * dirs + dir) * Bn + b) * H;
        for (int r = threadIdx.x; r < H; r += blockDim.x) {
          h[r] = hn[r];
          c[r] = cn[r];
          y[r] = hn[r];
        }
        __syncthreads();
      }
    }
    for (int b = 0; b < Bn; ++b)
      for (int r = threadIdx.x; r < H; r += blockDim.x) {
        if (Yh) Yh[((int64_t)dir * Bn + b) * H + r] = h[r];
        if (Yc) Yc[((int64_t)dir * Bn + b) * H + r] = c[r];
      }
    __syncthreads();
  }
}

bool data_ok(const Tensor* t, const char* op, const char* name) {
  if (!valid_tensor(t, op, name)) return false;
  if (tag_of(t) != 0) {
    fail(NNC_CUDA_ERR_UNSUPPORTED, op, "%s: storage tags are not supported here", name);
    return false;
  }
  return true;
}

int blocks_for(int64_t n) { return grid_for(n, kThreads, 8); }

}  // namespace
}  // namespace nnc

using namespace nnc;

extern "C" {

void nnc_cast(Tensor* input, Tensor* output, int to_dtype) {
  const char* op = "nnc_cast";
  OpScope scope(op);
  if (!data_ok(input, op, "input") || !data_ok(output, op, "output")) return;
  trace_io(tensor_bytes(input), tensor_bytes(output));
  const int64_t n = numel(input);  // the reference converts numel(input) elements
  if (n == 0) return;
  const bool src_bool = elem_type(input) == NNC_DTYPE_BOOL;
  cudaStream_t st = ctx().stream;
  // Plain copies of the reference: float -> float32, to float16 (4-byte
  // elements copied, a quirk kept), bool -> bool, unknown targets.
  size_t copy = 0;
  if (to_dtype == NNC_DTYPE_FLOAT32 && !src_bool) copy = (size_t)n * 4;
  else if (to_dtype == NNC_DTYPE_FLOAT16) copy = (size_t)n * 4;
  else if (to_dtype == NNC_DTYPE_BOOL && src_bool) copy = (size_t)n;
  else if (to_dtype != NNC_DTYPE_FLOAT32 && to_dtype != NNC_DTYPE_INT32 &&
           to_dtype != NNC_DTYPE_INT64 && to_dtype != NNC_DTYPE_BOOL)
    copy = (size_t)n * 4;
  if (copy) {
    check_cuda(cudaMemcpyAsync(output->data, input->data, copy, cudaMemcpyDeviceToDevice, st), op,
               "cudaMemcpyAsync");
    return;
  }
  cast_kernel<<<blocks_for(n), kThreads, 0, st>>>(input->data, output->data, n, to_dtype,
                                                 src_bool ? 1 : 0);
  check_launch(op);
}

static void compare_impl(Tensor* a, Tensor* b, Tensor* out, int kind, const char* op) {
  OpScope scope(op);
  if (!data_ok(a, op, "a") || !data_ok(b, op, "b") || !data_ok(out, op, "out")) return;
  trace_io(tensor_bytes(a) + tensor_bytes(b), tensor_bytes(out));
  const int64_t n = numel(out), an = numel(a), bn = numel(b);
  if (n == 0 || an == 0 || bn == 0) return;
  // Elements the reference writes: all n when each operand has n elements or
  // broadcasts over them, else min(n, a_n, b_n).
  int64_t w = n;
  const bool a_full = an == n, b_full = bn == n;
  if (!((a_full || b_full))) w = std::min(n, std::min(an, bn));
  cudaStream_t st = ctx().stream;
  if (kind == kEqual)
    cmp_kernel<kEqual><<<blocks_for(w), kThreads, 0, st>>>((const float*)a->data, (const float*)b->data,
                                                          (float*)out->data, w, an, bn);
  else
    cmp_kernel<kAnd><<<blocks_for(w), kThreads, 0, st>>>((const float*)a->data, (const float*)b->data,
                                                        (float*)out->data, w, an, bn);
  check_launch(op);
}

void nnc_equal(Tensor* a, Tensor* b, Tensor* out) { compare_impl(a, b, out, kEqual, "nnc_equal"); }
void nnc_and(Tensor* a, Tensor* b, Tensor* out) { compare_impl(a, b, out, kAnd, "nnc_and"); }

void nnc_greater(Tensor* a, Tensor* b, Tensor* out) {
  const char* op = "nnc_greater";
  OpScope scope(op);
  if (!data_ok(a, op, "a") || !data_ok(b, op, "b") || !data_ok(out, op, "out")) return;
  trace_io(tensor_bytes(a) + tensor_bytes(b), tensor_bytes(out));
  const int64_t n = numel(out), an = numel(a), bn = numel(b);
  if (n == 0) return;
  if (an == 0 || bn == 0) {
    fail(NNC_CUDA_ERR_INVALID, op, "empty operand");
    return;
  }
  greater_kernel<<<blocks_for(n), kThreads, 0, ctx().stream>>>(
      (const float*)a->data, (const float*)b->data, (uint8_t*)out->data, n, an, bn);
  check_launch(op);
}

void nnc_or(Tensor* a, Tensor* b, Tensor* out) {
  const char* op = "nnc_or";
  OpScope scope(op);
  if (!data_ok(a, op, "a") || !data_ok(b, op, "b") || !data_ok(out, op, "out")) return;
  trace_io(tensor_bytes(a) + tensor_bytes(b), tensor_bytes(out));
  const int64_t n = numel(out);
  if (n == 0) return;
  if (numel(a) < n || numel(b) < n) {
    fail(NNC_CUDA_ERR_INVALID, op, "operands shorter than the output");
    return;
  }
  or_kernel<<<blocks_for(n), kThreads, 0, ctx().stream>>>((const uint8_t*)a->data, (const uint8_t*)b->data,
                                                          (uint8_t*)out->data, n);
  check_launch(op);
}

void nnc_not(Tensor* input, Tensor* output) {
  const char* op = "nnc_not";
  OpScope scope(op);
  if (!data_ok(input, op, "input") || !data_ok(output, op, "output")) return;
  trace_io(tensor_bytes(input), tensor_bytes(output));
  const int64_t n = numel(output);
  if (n == 0) return;
  if (numel(input) < n) {
    fail(NNC_CUDA_ERR_INVALID, op, "input shorter than the output");
    return;
  }
  not_kernel<<<blocks_for(n), kThreads, 0, ctx().stream>>>((const uint8_t*)input->data,
                                                           (uint8_t*)output->data, n);
  check_launch(op);
}

void nnc_shape(Tensor* input, Tensor* output, int64_t* shape_data, int ndim) {
  const char* op = "nnc_shape";
  OpScope scope(op);
  if (!valid_tensor(output, op, "output")) return;
  if (ndim < 0 || ndim > 8) {
    fail(NNC_CUDA_ERR_INVALID, op, "ndim %d outside [0, 8]", ndim);
    return;
  }
  if (!shape_data && (!valid_tensor(input, op, "input") || input->ndim < ndim)) {
    fail(NNC_CUDA_ERR_INVALID, op, "input has fewer than %d dimensions", ndim);
    return;
  }
  if (ndim == 0) return;
  // The values (compile-time shape, else the input's host shape) are passed
  // by value to a one-thread-per-value kernel: no host buffer to outlive the
  // call, and the call can be captured into a graph.
  Dims8 v{};
  for (int i = 0; i < ndim; ++i) v.v[i] = shape_data ? shape_data[i] : input->shape[i];
  trace_io(0, (uint64_t)ndim * 8);
  write_i64_kernel<<<1, 32, 0, ctx().stream>>>((int64_t*)output->data, v, ndim);
  check_launch(op);
}

void nnc_constantofshape(Tensor* output, float value, int ndim) {
  const char* op = "nnc_constantofshape";
  OpScope scope(op);
  if (!valid_tensor(output, op, "output")) return;
  trace_io(0, tensor_bytes(output));
  const int64_t n = numel(output);
  if (n == 0) return;
  fill_kernel<<<blocks_for(n), kThreads, 0, ctx().stream>>>((float*)output->data, n, value);
  check_launch(op);
}

void nnc_expand(Tensor* input, Tensor* output, int64_t* shape, int ndim) {
  const char* op = "nnc_expand";
  OpScope scope(op);
  if (!data_ok(input, op, "input") || !data_ok(output, op, "output")) return;
  trace_io(tensor_bytes(input), tensor_bytes(output));
  const int64_t in_n = numel(input), out_n = numel(output);
  if (out_n == 0) return;
  if (in_n == 0) {
    fail(NNC_CUDA_ERR_INVALID, op, "empty input");
    return;
  }
  // ops.c:2633-2653: a copy when the sizes agree, else out[i] = in[i % in_n].
  modular_copy_kernel<float><<<blocks_for(out_n), kThreads, 0, ctx().stream>>>(
      (const float*)input->data, (float*)output->data, out_n, in_n);
  check_launch(op);
}

void nnc_tile(Tensor* input, Tensor* output, int64_t* repeats, int ndim) {
  const char* op = "nnc_tile";
  OpScope scope(op);
  if (!data_ok(input, op, "input") || !data_ok(output, op, "output")) return;
  trace_io(tensor_bytes(input), tensor_bytes(output));
  const int64_t n = numel(output);
  if (n == 0) return;
  if (!repeats) {  // ops.c:2271-2277: copy numel(output) elements
    check_cuda(cudaMemcpyAsync(output->data, input->data, (size_t)n * 4, cudaMemcpyDeviceToDevice,
                               ctx().stream),
               op, "cudaMemcpyAsync");
    return;
  }
  if (input->ndim < 1 || input->ndim > 8 || output->ndim < input->ndim || output->ndim > 8) {
    fail(NNC_CUDA_ERR_INVALID, op, "ranks %d -> %d are not supported", input->ndim, output->ndim);
    return;
  }
  TileGeom g{};
  g.out_ndim = output->ndim;
  g.in_ndim = input->ndim;
  for (int d = 0; d < output->ndim; ++d) g.out_shape[d] = output->shape[d];
  for (int d = 0; d < input->ndim; ++d) {
    g.in_shape[d] = input->shape[d];
    if (g.in_shape[d] <= 0) return;
  }
  g.in_stride[input->ndim - 1] = 1;
  for (int d = input->ndim - 2; d >= 0; --d) g.in_stride[d] = g.in_stride[d + 1] * input->shape[d + 1];
  tile_kernel<<<blocks_for(n), kThreads, 0, ctx().stream>>>((const float*)input->data,
                                                            (float*)output->data, n, g);
  check_launch(op);
}

void nnc_gather(Tensor* data, Tensor* indices, Tensor* output, int axis, int data_dtype) {
  const char* op = "nnc_gather";
  OpScope scope(op);
  if (!data_ok(data, op, "data") || !data_ok(indices, op, "indices") || !data_ok(output, op, "output"))
    return;
  trace_io(tensor_bytes(data) + tensor_bytes(indices), tensor_bytes(output));
  const int rank = data->ndim, irank = indices->ndim, orank = output->ndim;
  if (rank < 1 || rank > 8) {
    fail(NNC_CUDA_ERR_INVALID, op, "data rank %d", rank);
    return;
  }
  // Axis normalisation and clamping of ops.c:2720-2726.
  if (axis < 0) axis += rank;
  if (axis < 0) axis = 0;
  if (axis >= rank) axis = rank - 1;
  GatherArgs a{};
  a.axis = axis;
  a.out_n = numel(output);
  a.axis_extent = data->shape[axis];
  a.d0 = data->shape[0];
  a.d1 = rank > 1 ? data->shape[1] : 1;
  a.d2 = rank > 2 ? data->shape[2] : 1;
  a.o0 = orank > 0 ? output->shape[0] : 1;
  a.o1 = orank > 1 ? output->shape[1] : 1;
  a.o2 = orank > 2 ? output->shape[2] : 1;
  int kase = -1;
  const bool scalar = irank == 0 || (irank == 1 && indices->shape[0] == 1);
  if (scalar) {  // ops.c:2731-2850
    if (data_dtype == 1) {
      if (rank == 1) {
        kase = kG_I64Rank1Scalar;
      } else {
        kase = kG_I64Rows;
        a.copy = 1;
        for (int d = axis + 1; d < rank; ++d) a.copy *= data->shape[d];
      }
    } else if (rank == 1) {
      kase = kG_F32Rank1Scalar;
    } else if (rank == 2 && orank == 2) {
      kase = kG_F32Rank2Scalar;
    } else if (rank == 3) {
      if (axis == 0 && orank == 2) kase = kG_F32Rank3Axis0Out2;
      else if (axis == 0 && orank == 3) kase = kG_F32Rank3Axis0Out3;
      else if (axis == 1) kase = kG_F32Rank3Axis1;
      else if (axis == 2) kase = kG_F32Rank3Axis2;
    }
  }
  if (kase < 0 && irank == 1) {  // ops.c:2852-2894
    a.num_idx = indices->shape[0];
    if (data_dtype == 1 && rank == 1) kase = kG_I64Rank1List;
    else if (rank == 2) kase = kG_F32Rank2List;  // float copies, int64 data included
  }
  cudaStream_t st = ctx().stream;
  if (kase < 0) {  // ops.c:2896-2910: out[i] = data[i % numel(data)]
    const int64_t dn = numel(data);
    if (a.out_n == 0) return;
    if (dn == 0) {
      fail(NNC_CUDA_ERR_INVALID, op, "empty data");
      return;
    }
    if (data_dtype == 1)
      modular_copy_kernel<int64_t><<<blocks_for(a.out_n), kThreads, 0, st>>>(
          (const int64_t*)data->data, (int64_t*)output->data, a.out_n, dn);
    else
      modular_copy_kernel<float><<<blocks_for(a.out_n), kThreads, 0, st>>>(
          (const float*)data->data, (float*)output->data, a.out_n, dn);
    check_launch(op);
    return;
  }
  if (numel(indices) < 1 || a.axis_extent < 1) {
    fail(NNC_CUDA_ERR_INVALID, op, "empty indices or gathered axis");
    return;
  }
  a.kase = kase;
  gather_kernel<<<blocks_for(std::max<int64_t>(a.out_n, 1)), kThreads, 0, st>>>(
      data->data, (const int64_t*)indices->data, output->data, a);
  check_launch(op);
}

void nnc_batchnorm(Tensor* input, Tensor* scale, Tensor* bias, Tensor* mean, Tensor* var,
                   Tensor* output, float epsilon, int momentum) {
  // The reference's nnc_batchnorm (ops.c:2088-2093) is an empty TODO: it
  // writes nothing. Mirrored: the output is left as it is (nnc-py's flows
  // fold batch normalisation into the preceding convolution instead).
  OpScope scope("nnc_batchnorm");
  (void)input, (void)scale, (void)bias, (void)mean, (void)var, (void)output, (void)epsilon,
      (void)momentum;
}

void nnc_lstm(Tensor* X, Tensor* W, Tensor* R, Tensor* B, Tensor* Y, Tensor* Y_h, Tensor* Y_c,
              int direction, int hidden_size) {
  const char* op = "nnc_lstm";
  OpScope scope(op);
  if (!data_ok(X, op, "X") || !data_ok(W, op, "W") || !data_ok(R, op, "R") || !data_ok(Y, op, "Y"))
    return;
  if ((B && !data_ok(B, op, "B")) || (Y_h && !data_ok(Y_h, op, "Y_h")) ||
      (Y_c && !data_ok(Y_c, op, "Y_c")))
    return;
  if (X->ndim != 3 || hidden_size < 1) {
    fail(NNC_CUDA_ERR_INVALID, op, "X must be [seq, batch, input] and hidden_size positive");
    return;
  }
  trace_io(tensor_bytes(X) + tensor_bytes(W) + tensor_bytes(R) + tensor_bytes(B),
           tensor_bytes(Y) + tensor_bytes(Y_h) + tensor_bytes(Y_c));
  const int T = (int)X->shape[0], Bn = (int)X->shape[1], I = (int)X->shape[2], H = hidden_size;
  const int dirs = direction == 2 ? 2 : 1;
  const size_t smem = (size_t)4 * H * sizeof(float);
  if (smem > 200 * 1024) {
    fail(NNC_CUDA_ERR_UNSUPPORTED, op, "hidden_size %d: the state exceeds shared memory", H);
    return;
  }
  if ((int64_t)T * Bn == 0) return;
  if (smem > 48 * 1024 &&
      !check_cuda(cudaFuncSetAttribute(lstm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem),
                  op, "cudaFuncSetAttribute"))
    return;
  const int threads = H < 1024 ? ((H + 31) / 32) * 32 : 1024;
  lstm_kernel<<<1, threads, smem, ctx().stream>>>(
      (const float*)X->data, (const float*)W->data, (const float*)R->data,
      B ? (const float*)B->data : nullptr, (float*)Y->data, Y_h ? (float*)Y_h->data : nullptr,
      Y_c ? (float*)Y_c->data : nullptr, T, Bn, I, H, dirs);
  check_launch(op);
}

}  // extern "C"
