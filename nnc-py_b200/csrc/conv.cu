// 2-D convolution as an implicit GEMM on the sm_100a tensor cores.
//
//   D[m, co] = sum_k A[m, k] * W[co, k]      m  = (n, oh, ow) output pixel
//                                            k  = (kh, kw, ci) tap x channel
// Activations are read channels-last (NHWC, channels padded to a multiple
// of 4 = one 16-byte chunk), weights are packed [C_out][K_pad] with the same
// k order (K_pad a multiple of 32). NCHW tensors at the API are converted to
// NHWC in scratch memory; tensors tagged NNC_CUDA_TAG_NHWC are used in place.
//
// Kernel (persistent, one CTA per SM, 288 threads):
//   warps 0..3  producers: thread r gathers row r (one output pixel) of the
//               128 x 32 A tile with 16-byte cp.async (zero-fill for taps
//               that fall in the padding), written in the 128-byte swizzle
//               layout; thread 0 also TMA-loads the BN x 32 weight tile.
//               Arrival on the stage barrier is asynchronous
//               (cp.async.mbarrier.arrive.noinc), so producers run ahead.
//   warp 4      TMEM allocation + single-thread tcgen05.mma issue (kind::tf32,
//               M = 128, N = BN, 4 k-steps per stage; 3 MMAs per k-step in
//               3xTF32 mode), commits release ring slots and accumulators.
//   warps 5..8  epilogue: tcgen05.ld, + bias, (+ residual), activation, store
//               NHWC rows (16-byte vectors) or NCHW planes (coalesced across
//               the warp's 32 consecutive pixels).
//
// Reference semantics (ops.c:720-1050): window origin o*stride - pad with the
// top/left pad only, out-of-range taps contribute zero, output extent from
// output->shape, bias added before one rounding to fp32, then the activation
// (relu: v > 0 ? v : 0; sigmoid: 1 / (1 + expf(-v))).
#include <math.h>

#include "common.cuh"
#include "tc.cuh"

namespace nnc {
namespace {

constexpr int BM = 128;
constexpr int BK = 32;
constexpr int kProducerThreads = 128;
constexpr int kConvThreads = 288;

enum Act : int { kActNone = 0, kActRelu = 1, kActSigmoid = 2, kActAddRelu = 3 };

struct ConvArgs {
  // geometry
  int N, H, W, C4;  // input (NHWC, C4 channels incl. padding)
  int OH, OW, Cout;
  int KH, KW, sh, sw, ph, pw;
  int K;  // KH*KW*C4 (valid k), K_pad = kblocks*32
  int kblocks;
  int64_t M;  // N*OH*OW
  int m_tiles, n_tiles;
  int64_t tiles;
  const float* x_hi;  // NHWC input (hi plane in 3xTF32 mode)
  const float* x_lo;  // lo plane (3xTF32) or nullptr
  const float* bias;
  const float* residual;  // same layout as the output
  float* out;
  int out_nhwc;
  int act;
  int* err;
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return (uint8_t*)(((uintptr_t)p + 1023) & ~(uintptr_t)1023);
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(tc::smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

template <int BN, int SPLIT, int STAGES>
struct ConvCfg {
  static constexpr uint32_t A_BYTES = BM * BK * 4;
  static constexpr uint32_t B_BYTES = BN * BK * 4;
  static constexpr uint32_t STAGE_BYTES = SPLIT * (A_BYTES + B_BYTES);
  static constexpr uint32_t TMEM_COLS = 2 * BN;
  static constexpr size_t SMEM = (size_t)STAGES * STAGE_BYTES + 1024 + 256;
};

template <int BN, int SPLIT, int STAGES>
__global__ void __launch_bounds__(kConvThreads, 1)
    conv_tc_kernel(const __grid_constant__ CUtensorMap tmW0, const __grid_constant__ CUtensorMap tmW1,
                   const ConvArgs g) {
  using Cfg = ConvCfg<BN, SPLIT, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* done = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(&full[s], kProducerThreads + 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      tc::mbar_init(&tfull[a], 1);
      tc::mbar_init(&tempty[a], 4);
    }
    tc::mbar_init(done, 1);
    tc::fence_barrier_init();
    tc::prefetch_tmap(&tmW0);
    if (SPLIT == 2) tc::prefetch_tmap(&tmW1);
  }
  if (warp == 4) {
    tc::tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp < 4) {
    // ---------------- producers: im2col gather of A, TMA of W ----------------
    const int row = threadIdx.x;  // 0..127
    const int64_t OHW = (int64_t)g.OH * g.OW;
    const int taps = g.KH * g.KW;
    const bool chan32 = (g.C4 % 32) == 0;
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int64_t t = blockIdx.x; t < g.tiles && ok; t += gridDim.x) {
      const int mt = (int)(t / g.n_tiles), nt = (int)(t % g.n_tiles);
      const int64_t m = (int64_t)mt * BM + row;
      const bool row_ok = m < g.M;
      int n_img = 0, ih0 = 0, iw0 = 0;
      if (row_ok) {
        n_img = (int)(m / OHW);
        const int rem = (int)(m % OHW);
        ih0 = (rem / g.OW) * g.sh - g.ph;
        iw0 = (rem % g.OW) * g.sw - g.pw;
      }
      const int64_t img_off = (int64_t)n_img * g.H * g.W * g.C4;
      for (int kb = 0; kb < g.kblocks; ++kb) {
        if (!tc::mbar_wait(&empty[stage], phase ^ 1, g.err)) {
          ok = false;
          break;
        }
        uint8_t* s = smem + stage * Cfg::STAGE_BYTES;
        if (threadIdx.x == 0) {
          tc::mbar_arrive_expect_tx(&full[stage], SPLIT * Cfg::B_BYTES);
          uint8_t* sb = s + SPLIT * Cfg::A_BYTES;
          tc::tma_load_2d(sb, &tmW0, &full[stage], kb * BK, nt * BN);
          if (SPLIT == 2) tc::tma_load_2d(sb + Cfg::B_BYTES, &tmW1, &full[stage], kb * BK, nt * BN);
        }
        const uint32_t dst_row = tc::smem_u32(s) + row * 128;
        const int k0 = kb * BK;
        if (chan32) {
          const int tap = k0 / g.C4, c0 = k0 - tap * g.C4;
          const int ih = ih0 + tap / g.KW, iw = iw0 + tap % g.KW;
          const bool v = row_ok && tap < taps && ih >= 0 && ih < g.H && iw >= 0 && iw < g.W;
          const int64_t off = v ? img_off + ((int64_t)ih * g.W + iw) * g.C4 + c0 : 0;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint32_t d = dst_row + ((j ^ (row & 7)) << 4);
            cp_async16(d, g.x_hi + off + 4 * j, v ? 16u : 0u);
            if (SPLIT == 2) cp_async16(d + Cfg::A_BYTES, g.x_lo + off + 4 * j, v ? 16u : 0u);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int k = k0 + 4 * j;
            const int tap = k / g.C4, c = k - tap * g.C4;
            const int ih = ih0 + tap / g.KW, iw = iw0 + tap % g.KW;
            const bool v = row_ok && tap < taps && ih >= 0 && ih < g.H && iw >= 0 && iw < g.W;
            const int64_t off = v ? img_off + ((int64_t)ih * g.W + iw) * g.C4 + c : 0;
            const uint32_t d = dst_row + ((j ^ (row & 7)) << 4);
            cp_async16(d, g.x_hi + off, v ? 16u : 0u);
            if (SPLIT == 2) cp_async16(d + Cfg::A_BYTES, g.x_lo + off, v ? 16u : 0u);
          }
        }
        cp_async_arrive_noinc(&full[stage]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
    // Let every cp.async of this thread land before the CTA can exit.
    asm volatile("cp.async.wait_all;" ::: "memory");
  } else if (warp == 4) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc = tc::idesc_tf32(BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; t < g.tiles && ok; t += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t aphase = (local >> 1) & 1;
        if (!tc::mbar_wait(&tempty[acc], aphase ^ 1, g.err)) break;
        tc::tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < g.kblocks; ++kb) {
          if (!tc::mbar_wait(&full[stage], phase, g.err)) {
            ok = false;
            break;
          }
          // The A tile was written through the generic proxy (cp.async);
          // make it visible to the tensor core's async-proxy reads.
          fence_proxy_async_smem();
          tc::tc_fence_after();
          const uint32_t sa = tc::smem_u32(smem + stage * Cfg::STAGE_BYTES);
          const uint32_t sb = sa + SPLIT * Cfg::A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 8; ++k) {
            const uint64_t a0 = tc::desc_kmajor_sw128(sa + k * 32);
            const uint64_t b0 = tc::desc_kmajor_sw128(sb + k * 32);
            const uint32_t accum = (kb | k) != 0;
            if (SPLIT == 1) {
              tc::mma_tf32(d_tmem, a0, b0, idesc, accum);
            } else {
              const uint64_t a1 = tc::desc_kmajor_sw128(sa + Cfg::A_BYTES + k * 32);
              const uint64_t b1 = tc::desc_kmajor_sw128(sb + Cfg::B_BYTES + k * 32);
              tc::mma_tf32(d_tmem, a1, b0, idesc, accum);
              tc::mma_tf32(d_tmem, a0, b1, idesc, 1);
              tc::mma_tf32(d_tmem, a0, b0, idesc, 1);
            }
          }
          tc::mma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        tc::mma_commit(&tfull[acc]);
      }
      tc::mma_commit(done);
      tc::mbar_wait(done, 0, g.err);
    }
  } else {
    // ---------------- epilogue (warps 5..8) ----------------
    const int quad = warp & 3;
    const int64_t OHW = (int64_t)g.OH * g.OW;
    const bool vec = g.out_nhwc && (g.Cout % 4 == 0) && ((((uintptr_t)g.out) & 15) == 0) &&
                     (!g.residual || ((((uintptr_t)g.residual) & 15) == 0));
    int local = 0;
    for (int64_t t = blockIdx.x; t < g.tiles; t += gridDim.x, ++local) {
      const int mt = (int)(t / g.n_tiles), nt = (int)(t % g.n_tiles);
      const int acc = local & 1;
      const uint32_t aphase = (local >> 1) & 1;
      if (!tc::mbar_wait(&tfull[acc], aphase, g.err)) break;
      tc::tc_fence_after();
      const int64_t m = (int64_t)mt * BM + quad * 32 + lane;
      const bool row_ok = m < g.M;
      int64_t n_img = 0, p = 0;
      if (row_ok) {
        n_img = m / OHW;
        p = m % OHW;
      }
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 16) {
        uint32_t r[16];
        __syncwarp();  // tcgen05.ld is .sync.aligned: the warp must be converged
        tc::tmem_ld16(tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BN + c0, r);
        tc::tmem_ld_wait();
        const int co0 = nt * BN + c0;
        if (!row_ok || co0 >= g.Cout) continue;
        float v[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int co = co0 + j;
          float x = __uint_as_float(r[j]);
          if (g.bias && co < g.Cout) x = __fadd_rn(x, g.bias[co]);
          v[j] = x;
        }
        if (g.out_nhwc) {
          float* dst = g.out + m * g.Cout + co0;
          const float* res = g.residual ? g.residual + m * g.Cout + co0 : nullptr;
          if (vec && co0 + 16 <= g.Cout) {
#pragma unroll
            for (int j = 0; j < 16; j += 4) {
              float4 o = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
              if (g.act == kActAddRelu) {
                const float4 rr = *reinterpret_cast<const float4*>(res + j);
                o.x = __fadd_rn(o.x, rr.x);
                o.y = __fadd_rn(o.y, rr.y);
                o.z = __fadd_rn(o.z, rr.z);
                o.w = __fadd_rn(o.w, rr.w);
              }
              if (g.act == kActRelu || g.act == kActAddRelu) {
                o.x = o.x > 0.0f ? o.x : 0.0f;
                o.y = o.y > 0.0f ? o.y : 0.0f;
                o.z = o.z > 0.0f ? o.z : 0.0f;
                o.w = o.w > 0.0f ? o.w : 0.0f;
              } else if (g.act == kActSigmoid) {
                o.x = 1.0f / (1.0f + expf(-o.x));
                o.y = 1.0f / (1.0f + expf(-o.y));
                o.z = 1.0f / (1.0f + expf(-o.z));
                o.w = 1.0f / (1.0f + expf(-o.w));
              }
              *reinterpret_cast<float4*>(dst + j) = o;
            }
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              if (co0 + j >= g.Cout) break;
              float o = v[j];
              if (g.act == kActAddRelu) o = __fadd_rn(o, res[j]);
              if (g.act == kActRelu || g.act == kActAddRelu) o = o > 0.0f ? o : 0.0f;
              else if (g.act == kActSigmoid) o = 1.0f / (1.0f + expf(-o));
              dst[j] = o;
            }
          }
        } else {
          // NCHW: channel co of image n at plane offset p; lanes hold
          // consecutive pixels, so each store instruction is coalesced.
          float* dst = g.out + (n_img * g.Cout + co0) * OHW + p;
          const float* res = g.residual ? g.residual + (n_img * g.Cout + co0) * OHW + p : nullptr;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            if (co0 + j >= g.Cout) break;
            float o = v[j];
            if (g.act == kActAddRelu) o = __fadd_rn(o, res[(int64_t)j * OHW]);
            if (g.act == kActRelu || g.act == kActAddRelu) o = o > 0.0f ? o : 0.0f;
            else if (g.act == kActSigmoid) o = 1.0f / (1.0f + expf(-o));
            dst[(int64_t)j * OHW] = o;
          }
        }
      }
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&tempty[acc]);
    }
  }

  tc::tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// ------------------------------------------------------ layout kernels ----

// OIHW -> [plane][Cout][K_pad], k = (kh*KW + kw)*C4 + ci, zero padded.
// split: plane 0 = tf32(w), plane 1 = w - tf32(w); else plane 0 = w.
__global__ void __launch_bounds__(256) pack_weight_kernel(const float* __restrict__ w,
                                                          float* __restrict__ out, int Cout,
                                                          int Cin, int KH, int KW, int C4,
                                                          int Kpad, int split) {
  const int64_t total = (int64_t)Cout * Kpad;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int co = (int)(i / Kpad), k = (int)(i % Kpad);
    const int tap = k / C4, ci = k % C4;
    float v = 0.0f;
    if (tap < KH * KW && ci < Cin) v = w[(((int64_t)co * Cin + ci) * KH + tap / KW) * KW + tap % KW];
    if (split) {
      const float h = tc::to_tf32(v);
      out[i] = h;
      out[total + i] = v - h;
    } else {
      out[i] = v;
    }
  }
}

// NCHW [N][C][HW] -> NHWC [N][HW][C4] (channels >= C zero), optional hi/lo.
__global__ void __launch_bounds__(256) nchw_to_nhwc_pad_kernel(const float* __restrict__ x,
                                                               float* __restrict__ hi,
                                                               float* __restrict__ lo, int N, int C,
                                                               int64_t HW, int C4) {
  __shared__ float tile[32][33];
  const int64_t tiles_p = cdiv(HW, 32), tiles_c = cdiv(C4, 32);
  const int64_t per_img = tiles_p * tiles_c;
  for (int64_t t = blockIdx.x; t < (int64_t)N * per_img; t += gridDim.x) {
    const int64_t n = t / per_img;
    const int64_t tp = (t % per_img) / tiles_c, tcb = (t % per_img) % tiles_c;
    const int tx = threadIdx.x & 31;
    for (int j = threadIdx.x >> 5; j < 32; j += 8) {
      const int64_t c = tcb * 32 + j, pix = tp * 32 + tx;
      tile[j][tx] = (c < C && pix < HW) ? x[(n * C + c) * HW + pix] : 0.0f;
    }
    __syncthreads();
    for (int j = threadIdx.x >> 5; j < 32; j += 8) {
      const int64_t pix = tp * 32 + j, c = tcb * 32 + tx;
      if (pix < HW && c < C4) {
        const float v = tile[tx][j];
        const int64_t o = (n * HW + pix) * C4 + c;
        if (lo) {
          const float h = tc::to_tf32(v);
          hi[o] = h;
          lo[o] = v - h;
        } else {
          hi[o] = v;
        }
      }
    }
    __syncthreads();
  }
}

// NHWC (C channels) -> NHWC with C4 channels, optional hi/lo split.
__global__ void __launch_bounds__(256) nhwc_repack_kernel(const float* __restrict__ x,
                                                          float* __restrict__ hi,
                                                          float* __restrict__ lo, int64_t P, int C,
                                                          int C4) {
  const int64_t total = P * C4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t pix = i / C4;
    const int c = (int)(i % C4);
    const float v = c < C ? x[pix * C + c] : 0.0f;
    if (lo) {
      const float h = tc::to_tf32(v);
      hi[i] = h;
      lo[i] = v - h;
    } else {
      hi[i] = v;
    }
  }
}

// ------------------------------------------------------------------ host --

int kpad_of(int KH, int KW, int C4) { return (int)cdiv((int64_t)KH * KW * C4, BK) * BK; }

template <int BN, int SPLIT, int STAGES>
bool launch_conv(ConvArgs g, const float* w0, const float* w1, const char* op) {
  using Cfg = ConvCfg<BN, SPLIT, STAGES>;
  const int Kpad = g.kblocks * BK;
  CUtensorMap tw0, tw1;
  const uint64_t dims[2] = {(uint64_t)Kpad, (uint64_t)g.Cout};
  const uint64_t strides[1] = {(uint64_t)Kpad * 4};
  const uint32_t box[2] = {BK, BN};
  if (!encode_tmap_f32(&tw0, w0, 2, dims, strides, box, nullptr, op)) return false;
  tw1 = tw0;
  if (SPLIT == 2 && !encode_tmap_f32(&tw1, w1, 2, dims, strides, box, nullptr, op)) return false;
  g.n_tiles = (int)cdiv(g.Cout, BN);
  g.m_tiles = (int)cdiv(g.M, BM);
  g.tiles = (int64_t)g.m_tiles * g.n_tiles;
  auto kern = conv_tc_kernel<BN, SPLIT, STAGES>;
  static bool attr_set = false;
  if (!attr_set) {
    if (!check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)Cfg::SMEM),
                    op, "cudaFuncSetAttribute"))
      return false;
    attr_set = true;
  }
  const int grid = (int)(g.tiles < sm_count() ? g.tiles : sm_count());
  kern<<<grid, kConvThreads, Cfg::SMEM, ctx().stream>>>(tw0, tw1, g);
  return check_launch(op);
}

bool conv_f32(const Tensor* t, const char* op, const char* name) {
  if (!valid_tensor(t, op, name)) return false;
  if (elem_type(t) != NNC_DTYPE_FLOAT32) {
    fail(NNC_CUDA_ERR_UNSUPPORTED, op, "%s: only float32 is supported", name);
    return false;
  }
  return true;
}

void conv_impl(Tensor* input, Tensor* weight, Tensor* bias, Tensor* residual, Tensor* output,
               int KH, int KW, int sh, int sw, int ph, int pw, int act, const char* op) {
  if (!conv_f32(input, op, "input") || !conv_f32(weight, op, "weight") ||
      !conv_f32(output, op, "output"))
    return;
  if (bias && !conv_f32(bias, op, "bias")) return;
  if (residual && !conv_f32(residual, op, "residual")) return;
  if (input->ndim != 4 || weight->ndim != 4 || output->ndim != 4) {
    fail(NNC_CUDA_ERR_INVALID, op, "expected 4-D tensors");
    return;
  }
  const int N = (int)input->shape[0], C = (int)input->shape[1], H = (int)input->shape[2],
            W = (int)input->shape[3];
  const int Cout = (int)weight->shape[0];
  const int OH = (int)output->shape[2], OW = (int)output->shape[3];
  if (weight->shape[1] != C || weight->shape[2] != KH || weight->shape[3] != KW) {
    fail(NNC_CUDA_ERR_INVALID, op, "weight shape [%lld,%lld,%lld,%lld] does not match C=%d %dx%d",
         (long long)weight->shape[0], (long long)weight->shape[1], (long long)weight->shape[2],
         (long long)weight->shape[3], C, KH, KW);
    return;
  }
  if (output->shape[0] != N || output->shape[1] != Cout) {
    fail(NNC_CUDA_ERR_INVALID, op, "output N/C mismatch");
    return;
  }
  if (sh <= 0 || sw <= 0 || KH <= 0 || KW <= 0) {
    fail(NNC_CUDA_ERR_INVALID, op, "kernel and stride must be positive");
    return;
  }
  if (bias && numel(bias) < Cout) {
    fail(NNC_CUDA_ERR_INVALID, op, "bias has fewer than C_out elements");
    return;
  }
  if (residual && (numel(residual) != numel(output) || is_nhwc(residual) != is_nhwc(output))) {
    fail(NNC_CUDA_ERR_INVALID, op, "residual must match the output's shape and layout");
    return;
  }
  const int64_t M = (int64_t)N * OH * OW;
  if (M == 0 || Cout == 0) return;
  const bool split = ctx().precision == NNC_CUDA_PRECISION_3XTF32;
  const int C4 = (C + 3) & ~3;
  const int Kpad = kpad_of(KH, KW, C4);
  const bool packed = (tag_of(weight) & NNC_CUDA_TAG_PACKED_CONV) != 0;

  // Scratch: NHWC input planes (unless usable in place) + packed weights.
  const bool in_place = is_nhwc(input) && C4 == C && !split;
  const int64_t x_elems = (int64_t)N * H * W * C4;
  const int64_t w_elems = (int64_t)Cout * Kpad;
  size_t need = 0;
  if (!in_place) need += (size_t)(split ? 2 : 1) * x_elems * 4;
  if (!packed) need += (size_t)(split ? 2 : 1) * w_elems * 4;
  float* ws = need ? (float*)workspace(need + 256, op) : nullptr;
  if (need && !ws) return;
  float* cur = ws;

  const float* x_hi = (const float*)input->data;
  const float* x_lo = nullptr;
  if (!in_place) {
    float* hi = cur;
    float* lo = split ? cur + x_elems : nullptr;
    cur += (split ? 2 : 1) * x_elems;
    if (is_nhwc(input)) {
      nhwc_repack_kernel<<<grid_for(x_elems, 256, 8), 256, 0, ctx().stream>>>(
          (const float*)input->data, hi, lo, (int64_t)N * H * W, C, C4);
    } else {
      const int64_t tiles = (int64_t)N * cdiv((int64_t)H * W, 32) * cdiv(C4, 32);
      const int grid = (int)(tiles < (int64_t)sm_count() * 16 ? tiles : (int64_t)sm_count() * 16);
      nchw_to_nhwc_pad_kernel<<<grid, 256, 0, ctx().stream>>>((const float*)input->data, hi, lo, N,
                                                              C, (int64_t)H * W, C4);
    }
    if (!check_launch(op)) return;
    x_hi = hi;
    x_lo = lo;
  }
  const float* w0 = (const float*)weight->data;
  const float* w1 = w0 + w_elems;  // packed layout: [hi][lo]
  if (!packed) {
    float* wp = cur;
    pack_weight_kernel<<<grid_for(w_elems, 256, 8), 256, 0, ctx().stream>>>(
        (const float*)weight->data, wp, Cout, C, KH, KW, C4, Kpad, split ? 1 : 0);
    if (!check_launch(op)) return;
    w0 = wp;
    w1 = wp + w_elems;
  }

  ConvArgs g{};
  g.N = N;
  g.H = H;
  g.W = W;
  g.C4 = C4;
  g.OH = OH;
  g.OW = OW;
  g.Cout = Cout;
  g.KH = KH;
  g.KW = KW;
  g.sh = sh;
  g.sw = sw;
  g.ph = ph;
  g.pw = pw;
  g.K = KH * KW * C4;
  g.kblocks = Kpad / BK;
  g.M = M;
  g.x_hi = x_hi;
  g.x_lo = x_lo;
  g.bias = bias ? (const float*)bias->data : nullptr;
  g.residual = residual ? (const float*)residual->data : nullptr;
  g.out = (float*)output->data;
  g.out_nhwc = is_nhwc(output) ? 1 : 0;
  g.act = act;
  g.err = device_error_word();

  if (!split) {
    if (Cout > 128)
      launch_conv<256, 1, 4>(g, w0, nullptr, op);
    else if (Cout > 64)
      launch_conv<128, 1, 6>(g, w0, nullptr, op);
    else
      launch_conv<64, 1, 8>(g, w0, nullptr, op);
  } else {
    if (Cout > 128)
      launch_conv<256, 2, 2>(g, w0, w1, op);
    else if (Cout > 64)
      launch_conv<128, 2, 3>(g, w0, w1, op);
    else
      launch_conv<64, 2, 4>(g, w0, w1, op);
  }
}

}  // namespace
}  // namespace nnc

using namespace nnc;

extern "C" {

void nnc_conv(Tensor* input, Tensor* weight, Tensor* bias, Tensor* output, int kernel_h,
              int kernel_w, int stride_h, int stride_w, int pad_h, int pad_w) {
  OpScope s("nnc_conv");
  conv_impl(input, weight, bias, nullptr, output, kernel_h, kernel_w, stride_h, stride_w, pad_h,
            pad_w, kActNone, "nnc_conv");
}
void nnc_conv_relu(Tensor* input, Tensor* weight, Tensor* bias, Tensor* output, int kernel_h,
                   int kernel_w, int stride_h, int stride_w, int pad_h, int pad_w) {
  OpScope s("nnc_conv_relu");
  conv_impl(input, weight, bias, nullptr, output, kernel_h, kernel_w, stride_h, stride_w, pad_h,
            pad_w, kActRelu, "nnc_conv_relu");
}
void nnc_conv_sigmoid(Tensor* input, Tensor* weight, Tensor* bias, Tensor* output, int kernel_h,
                      int kernel_w, int stride_h, int stride_w, int pad_h, int pad_w) {
  OpScope s("nnc_conv_sigmoid");
  conv_impl(input, weight, bias, nullptr, output, kernel_h, kernel_w, stride_h, stride_w, pad_h,
            pad_w, kActSigmoid, "nnc_conv_sigmoid");
}

// 1x1: kernel 1 with the given stride/pad (ops.c:1217-1297).
void nnc_conv1x1(Tensor* input, Tensor* weight, Tensor* bias, Tensor* output, int stride_h,
                 int stride_w, int pad_h, int pad_w) {
  OpScope s("nnc_conv1x1");
  conv_impl(input, weight, bias, nullptr, output, 1, 1, stride_h, stride_w, pad_h, pad_w, kActNone,
            "nnc_conv1x1");
}
void nnc_conv_relu1x1(Tensor* input, Tensor* weight, Tensor* bias, Tensor* output, int stride_h,
                      int stride_w, int pad_h, int pad_w) {
  OpScope s("nnc_conv_relu1x1");
  conv_impl(input, weight, bias, nullptr, output, 1, 1, stride_h, stride_w, pad_h, pad_w, kActRelu,
            "nnc_conv_relu1x1");
}

// 3x3 stride 1 pad 1, output the input's size (ops.c:1052-1215; the
// reference rejects other output sizes, ops.c:1088-1092).
static bool same_size(Tensor* input, Tensor* output, const char* op) {
  if (!input || !output || !input->shape || !output->shape || input->ndim != 4 ||
      output->ndim != 4) {
    fail(NNC_CUDA_ERR_INVALID, op, "expected 4-D tensors");
    return false;
  }
  if (input->shape[2] != output->shape[2] || input->shape[3] != output->shape[3]) {
    fail(NNC_CUDA_ERR_INVALID, op, "expected same-padding output shape");
    return false;
  }
  return true;
}
void nnc_conv3x3_s1(Tensor* input, Tensor* weight, Tensor* bias, Tensor* output) {
  OpScope s("nnc_conv3x3_s1");
  if (!same_size(input, output, "nnc_conv3x3_s1")) return;
  conv_impl(input, weight, bias, nullptr, output, 3, 3, 1, 1, 1, 1, kActNone, "nnc_conv3x3_s1");
}
void nnc_conv_relu3x3_s1(Tensor* input, Tensor* weight, Tensor* bias, Tensor* output) {
  OpScope s("nnc_conv_relu3x3_s1");
  if (!same_size(input, output, "nnc_conv_relu3x3_s1")) return;
  conv_impl(input, weight, bias, nullptr, output, 3, 3, 1, 1, 1, 1, kActRelu,
            "nnc_conv_relu3x3_s1");
}

// 7x7 stride 2 pad 3 (ops.c:1336-1447).
void nnc_conv7x7_s2(Tensor* input, Tensor* weight, Tensor* bias, Tensor* output) {
  OpScope s("nnc_conv7x7_s2");
  conv_impl(input, weight, bias, nullptr, output, 7, 7, 2, 2, 3, 3, kActNone, "nnc_conv7x7_s2");
}
void nnc_conv_relu7x7_s2(Tensor* input, Tensor* weight, Tensor* bias, Tensor* output) {
  OpScope s("nnc_conv_relu7x7_s2");
  conv_impl(input, weight, bias, nullptr, output, 7, 7, 2, 2, 3, 3, kActRelu,
            "nnc_conv_relu7x7_s2");
}

void nnc_conv_add_relu(Tensor* input, Tensor* weight, Tensor* bias, Tensor* residual,
                       Tensor* output, int kernel_h, int kernel_w, int stride_h, int stride_w,
                       int pad_h, int pad_w) {
  OpScope s("nnc_conv_add_relu");
  if (!residual) {
    fail(NNC_CUDA_ERR_INVALID, "nnc_conv_add_relu", "NULL residual");
    return;
  }
  conv_impl(input, weight, bias, residual, output, kernel_h, kernel_w, stride_h, stride_w, pad_h,
            pad_w, kActAddRelu, "nnc_conv_add_relu");
}
void nnc_conv_add_relu1x1(Tensor* input, Tensor* weight, Tensor* bias, Tensor* residual,
                          Tensor* output, int stride_h, int stride_w, int pad_h, int pad_w) {
  OpScope s("nnc_conv_add_relu1x1");
  if (!residual) {
    fail(NNC_CUDA_ERR_INVALID, "nnc_conv_add_relu1x1", "NULL residual");
    return;
  }
  conv_impl(input, weight, bias, residual, output, 1, 1, stride_h, stride_w, pad_h, pad_w,
            kActAddRelu, "nnc_conv_add_relu1x1");
}
void nnc_conv_add_relu3x3_s1(Tensor* input, Tensor* weight, Tensor* bias, Tensor* residual,
                             Tensor* output) {
  OpScope s("nnc_conv_add_relu3x3_s1");
  if (!residual) {
    fail(NNC_CUDA_ERR_INVALID, "nnc_conv_add_relu3x3_s1", "NULL residual");
    return;
  }
  if (!same_size(input, output, "nnc_conv_add_relu3x3_s1")) return;
  conv_impl(input, weight, bias, residual, output, 3, 3, 1, 1, 1, 1, kActAddRelu,
            "nnc_conv_add_relu3x3_s1");
}

size_t nnc_cuda_prepacked_conv_weight_bytes(const Tensor* w) {
  if (!w || !w->shape || w->ndim != 4) return 0;
  const int C4 = ((int)w->shape[1] + 3) & ~3;
  return (size_t)2 * w->shape[0] * kpad_of((int)w->shape[2], (int)w->shape[3], C4) * 4;
}

int nnc_cuda_prepack_conv_weight(Tensor* w, void* dst, size_t dst_bytes) {
  const char* op = "nnc_cuda_prepack_conv_weight";
  OpScope s(op);
  if (!conv_f32(w, op, "weight")) return ctx().status;
  if (w->ndim != 4 || (tag_of(w) & NNC_CUDA_TAG_PACKED_CONV)) {
    fail(NNC_CUDA_ERR_INVALID, op, "expected an unpacked 4-D OIHW weight");
    return NNC_CUDA_ERR_INVALID;
  }
  const size_t need = nnc_cuda_prepacked_conv_weight_bytes(w);
  if (!dst || dst_bytes < need || !aligned16(dst)) {
    fail(NNC_CUDA_ERR_INVALID, op, "destination needs %zu bytes, 16-byte aligned", need);
    return NNC_CUDA_ERR_INVALID;
  }
  const int Cout = (int)w->shape[0], Cin = (int)w->shape[1], KH = (int)w->shape[2],
            KW = (int)w->shape[3];
  const int C4 = (Cin + 3) & ~3;
  const int Kpad = kpad_of(KH, KW, C4);
  const int64_t total = (int64_t)Cout * Kpad;
  pack_weight_kernel<<<grid_for(total, 256, 8), 256, 0, ctx().stream>>>(
      (const float*)w->data, (float*)dst, Cout, Cin, KH, KW, C4, Kpad, 1);
  if (!check_launch(op)) return ctx().status;
  w->data = dst;
  w->dtype = (nnc_dtype_t)((int)w->dtype | NNC_CUDA_TAG_PACKED_CONV);
  return NNC_CUDA_OK;
}

}  // extern "C"
