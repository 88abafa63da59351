// Element-wise operators: binary with the reference's modular suffix
// broadcast, unary activations/math, fused add+relu / add+sigmoid.
//
// HBM-bound: one read per input element and one write per output element,
// 128-bit vector accesses when every pointer is 16-byte aligned, grid-stride
// loops sized to a multiple of the SM count. Arithmetic is IEEE fp32 with no
// contraction (the file is built with -fmad=false), so add/sub/mul/div/relu/
// clip/abs/neg/pow are bit-identical to the reference's scalar C.
#include <math.h>

#include "common.cuh"

namespace nnc {
namespace {

enum Op : int {
  kAdd,
  kSub,
  kMul,
  kDiv,
  kAddRelu,
  kAddSigmoid,
  kRelu,
  kSigmoid,
  kTanh,
  kClip,
  kSqrt,
  kPow2,
  kExp,
  kLog,
  kAbs,
  kNeg,
};

// fmaxf / fminf as the reference binary computes them (ops.c:236, :2260):
// glibc returns the non-NaN operand when one is NaN and, for equal operands
// (+0 vs -0), the SECOND argument. Relu is written fmaxf(0.0f, x) in the
// reference but the compiled call passes x first, so relu(-0) = relu(NaN) =
// +0 — identical to x > 0 ? x : 0.
__device__ __forceinline__ float libm_fmaxf(float x, float y) {
  if (isnan(x)) return y;
  if (isnan(y)) return x;
  return (x > y) ? x : y;
}
__device__ __forceinline__ float libm_fminf(float x, float y) {
  if (isnan(x)) return y;
  if (isnan(y)) return x;
  return (x < y) ? x : y;
}

template <int OP>
__device__ __forceinline__ float binop(float a, float b) {
  if constexpr (OP == kAdd) return a + b;
  if constexpr (OP == kSub) return a - b;
  if constexpr (OP == kMul) return a * b;
  if constexpr (OP == kDiv) return a / b;
  if constexpr (OP == kAddRelu) {  // ops.c:3257-3261: s > 0 ? s : 0
    float s = a + b;
    return s > 0.0f ? s : 0.0f;
  }
  if constexpr (OP == kAddSigmoid) {  // ops.c:3313-3317
    float s = a + b;
    return 1.0f / (1.0f + expf(-s));
  }
  return 0.0f;
}

struct UnaryArgs {
  float lo, hi;  // clip bounds
};

template <int OP>
__device__ __forceinline__ float unop(float x, UnaryArgs p) {
  if constexpr (OP == kRelu) return x > 0.0f ? x : 0.0f;                 // ops.c:236
  if constexpr (OP == kSigmoid) return 1.0f / (1.0f + expf(-x));        // ops.c:246
  if constexpr (OP == kTanh) return tanhf(x);                           // ops.c:256
  if constexpr (OP == kClip) return libm_fminf(libm_fmaxf(x, p.lo), p.hi);  // ops.c:2260
  if constexpr (OP == kSqrt) return (x >= 0.0f) ? sqrtf(x) : __int_as_float(0x7fc00000);  // ops.c:2445
  if constexpr (OP == kPow2) return x * x;                              // ops.c:2459
  if constexpr (OP == kExp) return expf(x);                             // ops.c:2472
  if constexpr (OP == kLog) return (x > 0.0f) ? logf(x) : __int_as_float(0x7fc00000);  // ops.c:2487
  if constexpr (OP == kAbs) return fabsf(x);                            // ops.c:2500
  if constexpr (OP == kNeg) return -x;                                  // ops.c:2513
  return x;
}

// Index modes for a binary operand: identity (a[i]), scalar (a[0]),
// modular (a[i % len]).
enum Mode : int { kIdent = 0, kScalar = 1, kModular = 2 };

template <int OP, int AM, int BM>
__global__ void __launch_bounds__(256) binary_vec4_kernel(const float* __restrict__ a,
                                                          const float* __restrict__ b,
                                                          float* out, int64_t n4, int64_t a_len,
                                                          int64_t b_len) {
  // n4 = number of float4 groups; modular lengths are multiples of 4.
  const float4* a4 = reinterpret_cast<const float4*>(a);
  const float4* b4 = reinterpret_cast<const float4*>(b);
  float4* o4 = reinterpret_cast<float4*>(out);
  const float as = (AM == kScalar) ? a[0] : 0.0f;
  const float bs = (BM == kScalar) ? b[0] : 0.0f;
  for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < n4;
       g += (int64_t)gridDim.x * blockDim.x) {
    float4 va, vb;
    if constexpr (AM == kIdent) va = a4[g];
    else if constexpr (AM == kScalar) va = make_float4(as, as, as, as);
    else va = a4[g % (a_len >> 2)];
    if constexpr (BM == kIdent) vb = b4[g];
    else if constexpr (BM == kScalar) vb = make_float4(bs, bs, bs, bs);
    else vb = b4[g % (b_len >> 2)];
    float4 r;
    r.x = binop<OP>(va.x, vb.x);
    r.y = binop<OP>(va.y, vb.y);
    r.z = binop<OP>(va.z, vb.z);
    r.w = binop<OP>(va.w, vb.w);
    o4[g] = r;
  }
}

template <int OP>
__global__ void __launch_bounds__(256) binary_scalar_kernel(const float* __restrict__ a,
                                                            const float* __restrict__ b,
                                                            float* out, int64_t begin, int64_t n,
                                                            int64_t a_mod, int64_t b_mod) {
  // a_mod / b_mod: 0 = identity indexing, else index modulo that length.
  for (int64_t i = begin + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float va = a[a_mod ? i % a_mod : i];
    const float vb = b[b_mod ? i % b_mod : i];
    out[i] = binop<OP>(va, vb);
  }
}

template <int OP>
__global__ void __launch_bounds__(256) unary_kernel(const float* __restrict__ in, float* out,
                                                    int64_t n, UnaryArgs p, int vec) {
  if (vec) {
    const int64_t n4 = n >> 2;
    const float4* i4 = reinterpret_cast<const float4*>(in);
    float4* o4 = reinterpret_cast<float4*>(out);
    for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < n4;
         g += (int64_t)gridDim.x * blockDim.x) {
      float4 v = i4[g];
      v.x = unop<OP>(v.x, p);
      v.y = unop<OP>(v.y, p);
      v.z = unop<OP>(v.z, p);
      v.w = unop<OP>(v.w, p);
      o4[g] = v;
    }
    for (int64_t i = (n4 << 2) + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
      out[i] = unop<OP>(in[i], p);
  } else {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
      out[i] = unop<OP>(in[i], p);
  }
}

bool check_f32(const Tensor* t, const char* op, const char* name) {
  if (!valid_tensor(t, op, name)) return false;
  if (elem_type(t) != NNC_DTYPE_FLOAT32) {
    fail(NNC_CUDA_ERR_UNSUPPORTED, op, "%s: only float32 is supported (dtype %d)", name,
         elem_type(t));
    return false;
  }
  return true;
}

template <int OP, int AM, int BM>
void launch_vec(const float* a, const float* b, float* out, int64_t n4, int64_t al, int64_t bl) {
  const int grid = grid_for(n4, 256, 8);
  binary_vec4_kernel<OP, AM, BM><<<grid, 256, 0, ctx().stream>>>(a, b, out, n4, al, bl);
}

template <int OP>
void binary_dispatch(Tensor* a, Tensor* b, Tensor* out, const char* name) {
  OpScope scope(name);
  if (!check_f32(a, name, "a") || !check_f32(b, name, "b") || !check_f32(out, name, "out")) return;
  trace_io(tensor_bytes(a) + tensor_bytes(b), tensor_bytes(out));
  const int64_t n = numel(out), an = numel(a), bn = numel(b);
  if (n == 0) return;
  // Which elements the reference writes, and how each operand is indexed
  // (ops.c:82-118): all n with modular broadcast when the other operand has
  // exactly n elements, otherwise only the first min(n, a_n, b_n).
  int64_t count = n, a_mod = 0, b_mod = 0;
  if (an >= n && bn >= n) {
  } else if (bn == n && an < n) {
    a_mod = an;
  } else if (an == n && bn < n) {
    b_mod = bn;
  } else {
    count = n < an ? n : an;
    count = count < bn ? count : bn;
  }
  if ((a_mod && an == 0) || (b_mod && bn == 0)) {
    fail(NNC_CUDA_ERR_INVALID, name, "empty operand cannot broadcast to %lld elements",
         (long long)n);
    return;
  }
  if (count == 0) return;
  const float* pa = (const float*)a->data;
  const float* pb = (const float*)b->data;
  float* po = (float*)out->data;
  const bool aligned = aligned16(pa) && aligned16(pb) && aligned16(po);
  const bool a_vec = a_mod == 0 || a_mod == 1 || (a_mod % 4 == 0);
  const bool b_vec = b_mod == 0 || b_mod == 1 || (b_mod % 4 == 0);
  int64_t done = 0;
  if (aligned && a_vec && b_vec && count >= 4) {
    const int64_t n4 = count >> 2;
    const int am = a_mod == 0 ? kIdent : (a_mod == 1 ? kScalar : kModular);
    const int bm = b_mod == 0 ? kIdent : (b_mod == 1 ? kScalar : kModular);
    if (am == kIdent && bm == kIdent) launch_vec<OP, kIdent, kIdent>(pa, pb, po, n4, an, bn);
    else if (am == kScalar && bm == kIdent) launch_vec<OP, kScalar, kIdent>(pa, pb, po, n4, an, bn);
    else if (am == kIdent && bm == kScalar) launch_vec<OP, kIdent, kScalar>(pa, pb, po, n4, an, bn);
    else if (am == kModular && bm == kIdent) launch_vec<OP, kModular, kIdent>(pa, pb, po, n4, an, bn);
    else launch_vec<OP, kIdent, kModular>(pa, pb, po, n4, an, bn);
    done = n4 << 2;
    if (!check_launch(name)) return;
  }
  if (done < count) {
    const int grid = grid_for(count - done, 256, 8);
    binary_scalar_kernel<OP><<<grid, 256, 0, ctx().stream>>>(pa, pb, po, done, count, a_mod, b_mod);
    check_launch(name);
  }
}

template <int OP>
void unary_dispatch(Tensor* in, Tensor* out, const char* name, UnaryArgs p = {0.f, 0.f}) {
  OpScope scope(name);
  if (!check_f32(in, name, "input") || !check_f32(out, name, "output")) return;
  trace_io(tensor_bytes(in), tensor_bytes(out));
  // The reference iterates over numel(output) (ops.c:231).
  const int64_t n = numel(out);
  if (n == 0) return;
  if (numel(in) < n) {
    fail(NNC_CUDA_ERR_INVALID, name, "input has %lld elements, output %lld",
         (long long)numel(in), (long long)n);
    return;
  }
  const float* pi = (const float*)in->data;
  float* po = (float*)out->data;
  const int vec = aligned16(pi) && aligned16(po);
  const int grid = grid_for(vec ? (n >> 2) + 1 : n, 256, 8);
  unary_kernel<OP><<<grid, 256, 0, ctx().stream>>>(pi, po, n, p, vec);
  check_launch(name);
}

}  // namespace
}  // namespace nnc

using namespace nnc;

extern "C" {

void nnc_add(Tensor* a, Tensor* b, Tensor* out) { binary_dispatch<kAdd>(a, b, out, "nnc_add"); }
void nnc_sub(Tensor* a, Tensor* b, Tensor* out) { binary_dispatch<kSub>(a, b, out, "nnc_sub"); }
void nnc_mul(Tensor* a, Tensor* b, Tensor* out) { binary_dispatch<kMul>(a, b, out, "nnc_mul"); }
void nnc_div(Tensor* a, Tensor* b, Tensor* out) { binary_dispatch<kDiv>(a, b, out, "nnc_div"); }
void nnc_add_relu(Tensor* a, Tensor* b, Tensor* out) {
  binary_dispatch<kAddRelu>(a, b, out, "nnc_add_relu");
}
void nnc_add_sigmoid(Tensor* a, Tensor* b, Tensor* out) {
  binary_dispatch<kAddSigmoid>(a, b, out, "nnc_add_sigmoid");
}

void nnc_relu(Tensor* in, Tensor* out) { unary_dispatch<kRelu>(in, out, "nnc_relu"); }
void nnc_sigmoid(Tensor* in, Tensor* out) { unary_dispatch<kSigmoid>(in, out, "nnc_sigmoid"); }
void nnc_tanh(Tensor* in, Tensor* out) { unary_dispatch<kTanh>(in, out, "nnc_tanh"); }
void nnc_clip(Tensor* in, Tensor* out, float min_val, float max_val) {
  unary_dispatch<kClip>(in, out, "nnc_clip", UnaryArgs{min_val, max_val});
}
void nnc_sqrt(Tensor* in, Tensor* out) { unary_dispatch<kSqrt>(in, out, "nnc_sqrt"); }
void nnc_pow(Tensor* in, Tensor* out) { unary_dispatch<kPow2>(in, out, "nnc_pow"); }
void nnc_exp(Tensor* in, Tensor* out) { unary_dispatch<kExp>(in, out, "nnc_exp"); }
void nnc_log(Tensor* in, Tensor* out) { unary_dispatch<kLog>(in, out, "nnc_log"); }
void nnc_abs(Tensor* in, Tensor* out) { unary_dispatch<kAbs>(in, out, "nnc_abs"); }
void nnc_neg(Tensor* in, Tensor* out) { unary_dispatch<kNeg>(in, out, "nnc_neg"); }

}  // extern "C"
