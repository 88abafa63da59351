// 2-D convolution as an implicit GEMM on the sm_100a tensor cores.
//
//   D[m, co] = sum_k A[m, k] * W[co, k]      m = (n, oh, ow) output pixel
//                                            k = tap x input channel
// Weights are packed [C_out][K_pad] (K_pad a multiple of 32) in one of two k
// orders chosen from the weight shape (see weight_layout):
//   chunk mode   k = (kh, kw, c) with channels padded to a multiple of 4, read
//                NHWC: NNC_CUDA_TAG_NHWC inputs with C % 4 == 0 in place,
//                others (NCHW drop-in calls, the RGB model input) converted
//                in scratch memory first;
//   element mode (reductions of at most 64, e.g. LeNet's 1x5x5 conv):
//                k = (c, kh, kw), the OIHW order, read in place in either
//                layout.
//
// Kernel (persistent, one CTA per SM, 416 threads = 13 warps):
//   warps 0..3  producers. TMA modes (square windows, equal strides and pads;
//               the common case): thread 0 alone issues per stage one TMA
//               load of the BN x 32 weight tile and TMA im2col loads of the
//               128 x 32 activation tile from the NHWC input (one load of 32
//               channels into the 128-byte swizzle layout when C4 % 32 == 0,
//               eight loads of 4-channel core-matrix columns otherwise).
//               Gather modes (other windows, tiny reductions): all 128
//               threads gather the A tile with cp.async (zero fill for taps
//               in the padding). Chunk mode: 16-byte copies, eight
//               neighbouring threads per 128-byte row; each thread owns eight
//               rows whose base offsets and tap-validity masks are computed
//               once per tile and advances its (tap, channel) position
//               incrementally. Element mode: 4-byte copies with per-k offsets
//               from a shared-memory table. Arrival is asynchronous
//               (cp.async.mbarrier.arrive.noinc), so producers run ahead.
//   warp 4      TMEM allocation + single-thread tcgen05.mma issue (kind::tf32,
//               M = 128, N = BN, 4 k-steps per stage; 3 MMAs per k-step in
//               3xTF32 mode), commits release ring slots and accumulators.
//   warps 5..12 epilogue, two warps per TMEM lane quadrant, each taking
//               alternate 32-column blocks (tcgen05.ld of 16 columns at a
//               time); NHWC outputs are staged through a 32 x 33 shared tile
//               so bias, residual (prefetched before staging) and stores run
//               row-contiguously (eight lanes per 128-byte row); NCHW
//               outputs store per channel plane, coalesced across the warp's
//               32 consecutive pixels.
//
// Reference semantics (ops.c:720-1050): window origin o*stride - pad with the
// top/left pad only, out-of-range taps contribute zero, output extent from
// output->shape, bias added before one rounding to fp32, then the activation
// (relu: v > 0 ? v : 0; sigmoid: 1 / (1 + expf(-v))).
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "tc.cuh"

namespace nnc {
namespace {

constexpr int BM = 128;
constexpr int BK = 32;
constexpr int kProducerWarps = 4;
constexpr int kProducerThreads = 32 * kProducerWarps;
constexpr int kMmaWarp = kProducerWarps;
constexpr int kEpilogueWarps = 8;  // two per TMEM lane quadrant, splitting the columns
constexpr int kConvThreads = 32 * (kProducerWarps + 1 + kEpilogueWarps);
constexpr int kRowsPerThread = BM * 8 / kProducerThreads;  // chunk mode: 8
constexpr int kRowStep = kProducerThreads / 8;              // chunk mode: rows per pass
constexpr int kElemPerThread = BM * BK / kProducerThreads;  // element mode: 32

enum Act : int { kActNone = 0, kActRelu = 1, kActSigmoid = 2, kActAddRelu = 3 };

// How the A (activation) operand reaches shared memory (see the file comment).
//   kIm2col128: TMA im2col, C4 % 32 == 0: one load of 128 pixels x 32
//               channels per stage into the 128-byte swizzle layout;
//   kIm2col16:  TMA im2col, C4 % 4 == 0: eight loads of 128 pixels x 4
//               channels per stage, each a 2 KB column of 8-row x 16-byte core
//               matrices (K-major, no swizzle);
//   kChunk / kElement: cp.async gathers by the producer warps (windows the
//               im2col bounding box cannot describe, and tiny reductions).
//   kHalo:      stride-1 windows, C4 % 32 == 0: one TMA load of an input
//               window per 32-channel block, shared by every tap (see
//               conv_halo_kernel).
enum Mode : int { kChunk = 0, kElement = 1, kIm2col128 = 2, kIm2col16 = 3, kHalo = 4 };
constexpr int kMaxElementK = 64;  // K_pad limit of the element mode (see weight_layout)

struct ConvArgs {
  int mode;
  // geometry
  int N, H, W, C4;  // input; C4 = channels as stored (kChunk: padded to 4)
  int OH, OW, Cout;
  int KH, KW, sh, sw, ph, pw;
  int K;  // valid k extent (kChunk: KH*KW*C4, kElement: C*KH*KW)
  int kblocks;
  int64_t M;  // N*OH*OW
  int m_tiles, n_tiles;
  int64_t tiles;
  int tiles_x, tiles_y;  // kHalo: 8 x 32 output tiles per image row / column
  // Fused max pooling of the activated conv result (kHalo, one channel
  // tile): pooled extent, window, stride, top/left pad.
  int pool, PH, PW, pkh, pkw, psh, psw, pph, ppw;
  int64_t xs_n, xs_c, xs_h, xs_w;  // element-mode input strides (elements)
  const float* x_hi;  // input (hi plane in 3xTF32 mode)
  const float* x_lo;  // lo plane (3xTF32) or nullptr
  const float* bias;
  const float* residual;  // same layout as the output
  float* out;
  int out_nhwc;
  int act;
  int direct_epi;  // channels-last epilogues store from TMEM fragments (store_tile's `direct`)
  int* err;
  // Paired kernel, stream-K (sk_q > 0): tiles [0, sk_dp_tiles) run whole,
  // cluster by cluster; the k-block iterations of the other tiles are split
  // evenly over the clusters (sk_q each, one more for the first sk_r).
  int64_t sk_dp_tiles, sk_q, sk_r;
  float* sk_part;      // one slot of 2 x BM x BN partial sums per cluster
  unsigned* sk_count;  // one arrival counter per slot (zero between launches)
  // Halo kernel, GATHER: the original 3-channel input of a space-to-depth
  // conv (element strides), whose windows the kernel builds itself.
  const float* src;
  int src_H, src_W;
  int64_t src_sn, src_sc, src_sh, src_sw;
};

// Output-channel order of packed conv weights. When C_out is a multiple of
// 32, packed row 32 g + j holds channel 32 g + perm_col(j): the accumulator's
// TMEM column j then holds that channel, and a 16x256b TMEM load (thread t:
// columns 8 q + 2 (t & 3) + {0, 1}, q = 0..3) hands thread t channels
// 4 (t & 3) + {0..3} and 16 + 4 (t & 3) + {0..3}: two 16-byte runs, so four
// threads cover 64 contiguous bytes of a pixel and the epilogue's global
// accesses are 16 bytes wide. Column j = 8 q + 2 c + h -> 16 (q >> 1) + 4 c +
// 2 (q & 1) + h (a bijection of 0..31).
__host__ __device__ __forceinline__ int perm_col(int j) {
  const int q = j >> 3, c = (j >> 1) & 3, h = j & 1;
  return 16 * (q >> 1) + 4 * c + 2 * (q & 1) + h;
}
__host__ __device__ __forceinline__ bool perm_rows(int cout) { return cout % 32 == 0; }

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return (uint8_t*)(((uintptr_t)p + 1023) & ~(uintptr_t)1023);
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(tc::smem_u32(bar))
               : "memory");
}

// Epilogue staging: one 32 x 33 fp32 tile per epilogue warp.
constexpr int kStageCols = 32;
constexpr uint32_t kEpiBytes = kEpilogueWarps * 32 * (kStageCols + 1) * 4;

template <int BN, int SPLIT, int STAGES>
struct ConvCfg {
  static constexpr uint32_t A_BYTES = BM * BK * 4;
  static constexpr uint32_t B_BYTES = BN * BK * 4;
  static constexpr uint32_t STAGE_BYTES = SPLIT * (A_BYTES + B_BYTES);
  // Two accumulators; in 3xTF32 mode two chunk buffers plus the running sum
  // (tc::promote_chunk32), rounded up to a power of two.
  static constexpr uint32_t TMEM_COLS = SPLIT == 1 ? 2 * BN : (3 * BN <= 256 ? 256 : 512);
  static constexpr uint32_t EPI_OFF = STAGES * STAGE_BYTES;
  static constexpr uint32_t KTAB_OFF = EPI_OFF + kEpiBytes;
  static constexpr uint32_t BAR_OFF = KTAB_OFF + 2 * kMaxElementK * 4;
  static constexpr size_t SMEM = (size_t)BAR_OFF + 256 + 1024;
};

__device__ __forceinline__ float activate(float o, int act) {
  if (act == kActRelu || act == kActAddRelu) return o > 0.0f ? o : 0.0f;
  if (act == kActSigmoid) return 1.0f / (1.0f + expf(-o));
  return o;
}

// Epilogue of one accumulator tile for one warp: TMEM lanes [32 quad, +32)
// (the hardware's lane-quadrant rule) of the BN-column accumulator at TMEM
// column acc_col, 32-column chunks c0 = c_first, c_first + c_step, ... below
// BN. rows(r) maps accumulator row r (0..127) to its output pixel
// m = (n, oh, ow), or -1 when the row is padding. Column j of a chunk holds
// channel perm_col(j) when C_out is a multiple of 32 (the packed weights'
// row order), else channel j.
//
// `direct` (channels-last, C_out a multiple of 32, 16-byte aligned output
// and residual): a 16x256b TMEM load of 16 columns of one 16-lane half gives
// thread t rows (t >> 2) + 16 hb + 8 k, k = 0, 1, at channels 16 u +
// 4 (t & 3) + {0..3}; each run is stored (and its residual loaded) as one
// 16-byte access, four threads covering 64 contiguous bytes of a pixel. This
// path uses no shared memory and no shuffles, which the tensor pipe's operand
// reads starve while the next tile's MMAs run (measured under N = 64 MMAs: an
// 8 KB warp tile staged through shared memory takes ~12k cycles, stored from
// the fragments 2-4k). Otherwise the chunk is staged through a 32 x 33 shared
// tile and written row-contiguously (NHWC), or per channel plane (NCHW).
// DIRECT_CODE compiles the direct path in (the halo kernel; the im2col
// kernel's 13 warps leave it 128 registers per thread, too few for it).
// STAGED_CODE = false (an instance without a staging tile) compiles the
// staged and NCHW paths out; a call that would need them records
// NNC_CUDA_ERR_INVALID in the device error word and writes nothing (the host
// never routes one there).
template <int BN, bool DIRECT_CODE, class RowMap, bool STAGED_CODE = true>
__device__ __forceinline__ void store_tile(const ConvArgs& g, uint32_t tmem_base, uint32_t acc_col,
                                           int nt, int quad, int c_first, int c_step, int lane,
                                           float* stage_tile, bool vec_ok, bool bias_vec,
                                           const RowMap& rows, bool direct) {
  const int64_t OHW = (int64_t)g.OH * g.OW;
  const bool perm = perm_rows(g.Cout);
  if (!STAGED_CODE && !(DIRECT_CODE && g.out_nhwc && direct)) {
    if (lane == 0 && g.err) atomicExch(g.err, 1 /* NNC_CUDA_ERR_INVALID */);
    return;
  }
  if (DIRECT_CODE && g.out_nhwc && direct) {
    const bool add = g.act == kActAddRelu;
    const bool relu = add || g.act == kActRelu;
#pragma unroll 1
    for (int c0 = c_first; c0 < BN; c0 += c_step) {
      const int co0 = nt * BN + c0;
      if (co0 >= g.Cout) continue;  // warp-uniform; C_out % 32 == 0: whole chunks
      const int cb = co0 + 4 * (lane & 3);  // channels cb + 16 u + {0..3}, u = 0, 1
      int64_t m[4];  // rows (t >> 2) + 8 k
#pragma unroll
      for (int k = 0; k < 4; ++k) m[k] = rows(quad * 32 + (lane >> 2) + 8 * k);
      // The chunk's residual runs and its four TMEM loads are all in flight
      // before the one wait: one memory round trip per chunk.
      float4 rv[4][2];
      if (add) {
#pragma unroll
        for (int k = 0; k < 4; ++k)
#pragma unroll
          for (int u = 0; u < 2; ++u)
            rv[k][u] = m[k] >= 0
                           ? __ldg(reinterpret_cast<const float4*>(g.residual + m[k] * g.Cout + cb + 16 * u))
                           : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      uint32_t r[4][8];  // [2 hb + u]: 16 columns c0 + 16 u of lanes + 16 hb
      __syncwarp();      // tcgen05.ld is .sync.aligned: the warp must be converged
#pragma unroll
      for (int hb = 0; hb < 2; ++hb)
#pragma unroll
        for (int u = 0; u < 2; ++u)
          tc::tmem_ld_16x256b_x2(
              tmem_base + ((uint32_t)(quad * 32 + 16 * hb) << 16) + acc_col + c0 + 16 * u,
              r[2 * hb + u]);
      float4 bv[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        bv[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (g.bias) {
          const float* bp = g.bias + cb + 16 * u;
          bv[u] = bias_vec ? __ldg(reinterpret_cast<const float4*>(bp))
                           : make_float4(__ldg(bp), __ldg(bp + 1), __ldg(bp + 2), __ldg(bp + 3));
        }
      }
      tc::tmem_ld_wait();
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (m[k] < 0) continue;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          // Row k is lane (t >> 2) + 8 (k & 1) of half k >> 1: registers
          // 2 (k & 1) + {0, 1} (columns 2 c + {0, 1}) and 4 + 2 (k & 1) + {0, 1}
          // (columns 8 + 2 c + {0, 1}) of load 2 (k >> 1) + u.
          const uint32_t* q = r[2 * (k >> 1) + u];
          const int i = 2 * (k & 1);
          float4 o = make_float4(__fadd_rn(__uint_as_float(q[i]), bv[u].x),
                                 __fadd_rn(__uint_as_float(q[i + 1]), bv[u].y),
                                 __fadd_rn(__uint_as_float(q[4 + i]), bv[u].z),
                                 __fadd_rn(__uint_as_float(q[4 + i + 1]), bv[u].w));
          if (add) {
            o.x = __fadd_rn(o.x, rv[k][u].x);
            o.y = __fadd_rn(o.y, rv[k][u].y);
            o.z = __fadd_rn(o.z, rv[k][u].z);
            o.w = __fadd_rn(o.w, rv[k][u].w);
          }
          if (relu) {
            o.x = o.x > 0.0f ? o.x : 0.0f;
            o.y = o.y > 0.0f ? o.y : 0.0f;
            o.z = o.z > 0.0f ? o.z : 0.0f;
            o.w = o.w > 0.0f ? o.w : 0.0f;
          } else {
            o.x = activate(o.x, g.act);
            o.y = activate(o.y, g.act);
            o.z = activate(o.z, g.act);
            o.w = activate(o.w, g.act);
          }
          *reinterpret_cast<float4*>(g.out + m[k] * g.Cout + cb + 16 * u) = o;
        }
      }
    }
    return;
  }
  if constexpr (STAGED_CODE) {
#pragma unroll 1
  for (int c0 = c_first; c0 < BN; c0 += c_step) {
    const int co0 = nt * BN + c0;
    if (co0 >= g.Cout) continue;  // warp-uniform: no TMEM load is skipped by part of a warp
    const uint32_t taddr = tmem_base + ((uint32_t)(quad * 32) << 16) + acc_col + c0;
    if (g.out_nhwc) {
      // Stage the 32 x 32 block, then write it row-contiguously: eight lanes
      // cover one 128-byte row segment (channels co .. co + 3), a warp four
      // rows. Channels cl + {0, 1} and cl + {2, 3} sit at staged columns
      // sa + {0, 1} and sb + {0, 1} (perm_col inverted: 16 u + 2 c and + 8,
      // cl = 16 u + 4 c).
      const int cl = (lane & 7) * 4;  // channel offset within the block
      const int co = co0 + cl;
      const int sa = perm ? 16 * ((lane & 7) >> 2) + 2 * (lane & 3) : cl;
      const int sb = perm ? sa + 8 : cl + 2;
      // 16-byte row accesses need C_out % 4 == 0 and aligned bases
      // (vec_ok); otherwise the per-element path below is taken.
      const bool col_ok = vec_ok && co + 3 < g.Cout;
      // Issue this chunk's residual loads first so their latency overlaps
      // the staging below.
      float4 rv[8];
      if (g.act == kActAddRelu && col_ok) {
#pragma unroll
        for (int it = 0; it < 8; ++it) {
          const int64_t m = rows(quad * 32 + (lane >> 3) + 4 * it);
          rv[it] = m >= 0 ? *reinterpret_cast<const float4*>(g.residual + m * g.Cout + co)
                          : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
#pragma unroll
      for (int h16 = 0; h16 < 2; ++h16) {
        uint32_t r[16];
        __syncwarp();  // tcgen05.ld is .sync.aligned: the warp must be converged
        tc::tmem_ld16(taddr + 16 * h16, r);
        tc::tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j)
          stage_tile[lane * (kStageCols + 1) + 16 * h16 + j] = __uint_as_float(r[j]);
      }
      __syncwarp();
      float4 bv = make_float4(0.f, 0.f, 0.f, 0.f);
      if (g.bias) {
        if (col_ok && bias_vec) {
          bv = *reinterpret_cast<const float4*>(g.bias + co);
        } else {
          bv.x = co < g.Cout ? g.bias[co] : 0.f;
          bv.y = co + 1 < g.Cout ? g.bias[co + 1] : 0.f;
          bv.z = co + 2 < g.Cout ? g.bias[co + 2] : 0.f;
          bv.w = co + 3 < g.Cout ? g.bias[co + 3] : 0.f;
        }
      }
      if (col_ok) {
        // Vector path, unrolled (rv stays in registers); the activation is
        // decided once per chunk so the body stays short.
        const bool add = g.act == kActAddRelu;
        const bool relu = add || g.act == kActRelu;
        const bool sig = g.act == kActSigmoid;
#pragma unroll
        for (int it = 0; it < 8; ++it) {
          const int rr = (lane >> 3) + 4 * it;
          const int64_t m = rows(quad * 32 + rr);
          if (m < 0) continue;
          const float* srow = stage_tile + rr * (kStageCols + 1);
          float4 o = make_float4(__fadd_rn(srow[sa], bv.x), __fadd_rn(srow[sa + 1], bv.y),
                                 __fadd_rn(srow[sb], bv.z), __fadd_rn(srow[sb + 1], bv.w));
          if (add) {
            o.x = __fadd_rn(o.x, rv[it].x);
            o.y = __fadd_rn(o.y, rv[it].y);
            o.z = __fadd_rn(o.z, rv[it].z);
            o.w = __fadd_rn(o.w, rv[it].w);
          }
          if (relu) {
            o.x = o.x > 0.0f ? o.x : 0.0f;
            o.y = o.y > 0.0f ? o.y : 0.0f;
            o.z = o.z > 0.0f ? o.z : 0.0f;
            o.w = o.w > 0.0f ? o.w : 0.0f;
          } else if (sig) {
            o.x = activate(o.x, kActSigmoid);
            o.y = activate(o.y, kActSigmoid);
            o.z = activate(o.z, kActSigmoid);
            o.w = activate(o.w, kActSigmoid);
          }
          *reinterpret_cast<float4*>(g.out + m * g.Cout + co) = o;
        }
      } else {
        // Per-element path: C_out % 4 != 0, unaligned bases, ragged last columns.
#pragma unroll 1
        for (int it = 0; it < 8; ++it) {
          const int rr = (lane >> 3) + 4 * it;
          const int64_t m = rows(quad * 32 + rr);
          if (m < 0) continue;
          const float* srow = stage_tile + rr * (kStageCols + 1);
          const float bq[4] = {bv.x, bv.y, bv.z, bv.w};
          for (int q = 0; q < 4 && co + q < g.Cout; ++q) {
            float v = __fadd_rn(srow[q < 2 ? sa + q : sb + q - 2], bq[q]);
            if (g.act == kActAddRelu) v = __fadd_rn(v, g.residual[m * g.Cout + co + q]);
            g.out[m * g.Cout + co + q] = activate(v, g.act);
          }
        }
      }
      __syncwarp();
    } else {
      // NCHW: channel c of image n at plane offset p; lanes hold
      // consecutive pixels, so each store instruction is coalesced.
      const int64_t m = rows(quad * 32 + lane);
      const int64_t n_img = m / OHW, p = m - n_img * OHW;
#pragma unroll
      for (int h16 = 0; h16 < 2; ++h16) {
        uint32_t r[16];
        __syncwarp();  // tcgen05.ld is .sync.aligned: the warp must be converged
        tc::tmem_ld16(taddr + 16 * h16, r);
        tc::tmem_ld_wait();
        if (m >= 0) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int c = co0 + (perm ? perm_col(16 * h16 + j) : 16 * h16 + j);
            if (c >= g.Cout) break;  // (unpermuted chunks end at the last channel)
            float o = __uint_as_float(r[j]);
            if (g.bias) o = __fadd_rn(o, g.bias[c]);
            const int64_t off = (n_img * g.Cout + c) * OHW + p;
            if (g.act == kActAddRelu) o = __fadd_rn(o, g.residual[off]);
            g.out[off] = activate(o, g.act);
          }
        }
      }
    }
  }
  }  // STAGED_CODE
}

// Row maps of the two tile shapes: a run of 128 consecutive output pixels,
// and an 8-wide x 16-tall block of one image (row r = 8 y + x).
struct LinearRows {
  int64_t m0, M;
  __device__ __forceinline__ int64_t operator()(int r) const { return m0 + r < M ? m0 + r : -1; }
};
struct BlockRows {
  int64_t img0;  // n * OH * OW
  int y0, x0, OH, OW;
  __device__ __forceinline__ int64_t operator()(int r) const {
    const int y = y0 + (r >> 3), x = x0 + (r & 7);
    return (y < OH && x < OW) ? img0 + (int64_t)y * OW + x : -1;
  }
};

template <int BN, int SPLIT, int STAGES>
__global__ void __launch_bounds__(kConvThreads, 1)
    conv_tc_kernel(const __grid_constant__ CUtensorMap tmW0, const __grid_constant__ CUtensorMap tmW1,
                   const __grid_constant__ CUtensorMap tmX0, const __grid_constant__ CUtensorMap tmX1,
                   const ConvArgs g) {
  using Cfg = ConvCfg<BN, SPLIT, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  pdl_trigger();
  uint8_t* smem = align1024(smem_raw);
  float* epi = reinterpret_cast<float*>(smem + Cfg::EPI_OFF);
  int* ktab_off = reinterpret_cast<int*>(smem + Cfg::KTAB_OFF);
  int* ktab_hw = ktab_off + kMaxElementK;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::BAR_OFF);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* done = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool tma_a = g.mode == kIm2col128 || g.mode == kIm2col16;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      // TMA feeding: one expect_tx arrival; gathers: every producer thread
      // arrives (cp.async.mbarrier.arrive.noinc) plus the weight TMA.
      tc::mbar_init(&full[s], tma_a ? 1 : kProducerThreads + 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      tc::mbar_init(&tfull[a], 1);
      tc::mbar_init(&tempty[a], kEpilogueWarps);
    }
    tc::mbar_init(done, 1);
    tc::fence_barrier_init();
    tc::prefetch_tmap(&tmW0);
    if (SPLIT == 2) tc::prefetch_tmap(&tmW1);
    if (tma_a) {
      tc::prefetch_tmap(&tmX0);
      if (SPLIT == 2) tc::prefetch_tmap(&tmX1);
    }
  }
  if (g.mode == kElement) {
    // k -> (element offset from the window origin, kh << 16 | kw); -1 past K.
    const int taps = g.KH * g.KW;
    for (int k = threadIdx.x; k < g.kblocks * BK; k += blockDim.x) {
      if (k < g.K) {
        const int c = k / taps, t = k - c * taps, kh = t / g.KW, kw = t - kh * g.KW;
        ktab_off[k] = (int)(c * g.xs_c + kh * g.xs_h + kw * g.xs_w);
        ktab_hw[k] = (kh << 16) | kw;
      } else {
        ktab_off[k] = 0;
        ktab_hw[k] = -1;
      }
    }
  }
  if (warp == kMmaWarp) {
    tc::tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // the previous kernel's outputs are complete from here on

  if (tma_a && warp < kProducerWarps) {
    // ---------------- producer (one thread): TMA im2col of A, TMA of W ----------------
    if (threadIdx.x == 0) {
      const int64_t OHW = (int64_t)g.OH * g.OW;
      const int taps = g.KH * g.KW;
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int64_t tile = blockIdx.x; tile < g.tiles && ok; tile += gridDim.x) {
        const int mt = (int)(tile / g.n_tiles), nt = (int)(tile % g.n_tiles);
        // Window origin of the tile's first output pixel: the im2col
        // traversal continues from there in (n, oh, ow) order.
        const int64_t m0 = (int64_t)mt * BM;
        const int n0 = (int)(m0 / OHW);
        const int rem = (int)(m0 - (int64_t)n0 * OHW);
        const int w0 = (rem % g.OW) * g.sw - g.pw, h0 = (rem / g.OW) * g.sh - g.ph;
        for (int kb = 0; kb < g.kblocks; ++kb) {
          if (!tc::mbar_wait(&empty[stage], phase ^ 1, g.err)) {
            ok = false;
            break;
          }
          uint8_t* s = smem + stage * Cfg::STAGE_BYTES;
          tc::mbar_arrive_expect_tx(&full[stage], Cfg::STAGE_BYTES);
          uint8_t* sb = s + SPLIT * Cfg::A_BYTES;
          tc::tma_load_2d(sb, &tmW0, &full[stage], kb * BK, nt * BN);
          if (SPLIT == 2) tc::tma_load_2d(sb + Cfg::B_BYTES, &tmW1, &full[stage], kb * BK, nt * BN);
          if (g.mode == kIm2col128) {
            const int k0 = kb * BK, tap = k0 / g.C4, c0 = k0 - tap * g.C4;
            const uint16_t kh = (uint16_t)(tap / g.KW), kw = (uint16_t)(tap % g.KW);
            tc::tma_load_im2col_4d(s, &tmX0, &full[stage], c0, w0, h0, n0, kw, kh);
            if (SPLIT == 2)
              tc::tma_load_im2col_4d(s + Cfg::A_BYTES, &tmX1, &full[stage], c0, w0, h0, n0, kw, kh);
          } else {
#pragma unroll 1
            for (int j = 0; j < 8; ++j) {
              // k = kb*32 + 4j -> (tap, channel group); past the last tap the
              // channel coordinate C4 is out of range, so the column is zeros.
              const int k = kb * BK + 4 * j;
              int tap = k / g.C4, c0 = k - tap * g.C4;
              if (tap >= taps) {
                tap = 0;
                c0 = g.C4;
              }
              const uint16_t kh = (uint16_t)(tap / g.KW), kw = (uint16_t)(tap % g.KW);
              tc::tma_load_im2col_4d(s + j * 2048, &tmX0, &full[stage], c0, w0, h0, n0, kw, kh);
              if (SPLIT == 2)
                tc::tma_load_im2col_4d(s + Cfg::A_BYTES + j * 2048, &tmX1, &full[stage], c0, w0, h0,
                                       n0, kw, kh);
            }
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Let the last issued loads land before the CTA can exit.
      if (ok) {
        for (int q = 0; q < STAGES; ++q) {
          if (stage == 0) {
            stage = STAGES;
            phase ^= 1;
          }
          --stage;
          tc::mbar_wait(&full[stage], phase, g.err);
        }
      }
    }
  } else if (warp < kProducerWarps) {
    // ---------------- producers: im2col gather of A, TMA of W ----------------
    const int t = threadIdx.x;  // 0..kProducerThreads-1
    const int64_t OHW = (int64_t)g.OH * g.OW;
    const int taps = g.KH * g.KW;
    const bool use_mask = taps <= 64;
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int64_t tile = blockIdx.x; tile < g.tiles && ok; tile += gridDim.x) {
      const int mt = (int)(tile / g.n_tiles), nt = (int)(tile % g.n_tiles);
      if (g.mode == kChunk) {
        // Thread t copies chunk j = t & 7 (channels 4j..4j+3 of the stage's
        // 32) of rows r_i = (t >> 3) + kRowStep * i.
        const int j = t & 7;
        int ih0[kRowsPerThread], iw0[kRowsPerThread];
        int64_t base[kRowsPerThread];
        uint64_t mask[kRowsPerThread];
#pragma unroll
        for (int i = 0; i < kRowsPerThread; ++i) {
          const int64_t m = (int64_t)mt * BM + (t >> 3) + kRowStep * i;
          mask[i] = 0;
          ih0[i] = -(1 << 28);
          iw0[i] = 0;
          base[i] = 0;
          if (m < g.M) {
            const int64_t n_img = m / OHW;
            const int rem = (int)(m - n_img * OHW);
            ih0[i] = (rem / g.OW) * g.sh - g.ph;
            iw0[i] = (rem % g.OW) * g.sw - g.pw;
            base[i] = (n_img * g.H * g.W + (int64_t)ih0[i] * g.W + iw0[i]) * g.C4;
            if (use_mask) {
              for (int kh = 0; kh < g.KH; ++kh) {
                if ((unsigned)(ih0[i] + kh) >= (unsigned)g.H) continue;
                for (int kw = 0; kw < g.KW; ++kw)
                  if ((unsigned)(iw0[i] + kw) < (unsigned)g.W) mask[i] |= 1ull << (kh * g.KW + kw);
              }
            }
          }
        }
        // This thread's chunk position: k = kb * 32 + 4j -> (tap, channel).
        int tap = (4 * j) / g.C4, c = 4 * j - tap * g.C4;
        int kh = tap / g.KW, kw = tap - kh * g.KW;
        int64_t toff = ((int64_t)kh * g.W + kw) * g.C4;
        for (int kb = 0; kb < g.kblocks; ++kb) {
          if (!tc::mbar_wait(&empty[stage], phase ^ 1, g.err)) {
            ok = false;
            break;
          }
          uint8_t* s = smem + stage * Cfg::STAGE_BYTES;
          if (t == 0) {
            tc::mbar_arrive_expect_tx(&full[stage], SPLIT * Cfg::B_BYTES);
            uint8_t* sb = s + SPLIT * Cfg::A_BYTES;
            tc::tma_load_2d(sb, &tmW0, &full[stage], kb * BK, nt * BN);
            if (SPLIT == 2) tc::tma_load_2d(sb + Cfg::B_BYTES, &tmW1, &full[stage], kb * BK, nt * BN);
          }
          const bool tap_ok = tap < taps;
          const uint32_t sbase = tc::smem_u32(s);
#pragma unroll
          for (int i = 0; i < kRowsPerThread; ++i) {
            const int r = (t >> 3) + kRowStep * i;
            bool v;
            if (use_mask) {
              v = tap_ok && ((mask[i] >> tap) & 1ull);
            } else {
              v = tap_ok && (unsigned)(ih0[i] + kh) < (unsigned)g.H &&
                  (unsigned)(iw0[i] + kw) < (unsigned)g.W;
            }
            const int64_t off = v ? base[i] + toff + c : 0;
            const uint32_t d = sbase + r * 128 + ((j ^ (r & 7)) << 4);
            cp_async16(d, g.x_hi + off, v ? 16u : 0u);
            if (SPLIT == 2) cp_async16(d + Cfg::A_BYTES, g.x_lo + off, v ? 16u : 0u);
          }
          cp_async_arrive_noinc(&full[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
          // Advance by 32 channels (several taps when C4 < 32).
          c += BK;
          while (c >= g.C4 && tap < taps) {
            c -= g.C4;
            ++tap;
            if (++kw == g.KW) {
              kw = 0;
              ++kh;
            }
            toff = ((int64_t)kh * g.W + kw) * g.C4;
          }
        }
      } else {
        // Element mode: thread t copies k values [kElemPerThread * h,
        // kElemPerThread * (h + 1)) of row r = t % BM of each 32-wide stage,
        // h = t / BM.
        const int r = t % BM, h = t / BM;
        const int64_t m = (int64_t)mt * BM + r;
        int ih0 = -(1 << 28), iw0 = 0;
        int64_t rbase = 0;
        if (m < g.M) {
          const int64_t n_img = m / OHW;
          const int rem = (int)(m - n_img * OHW);
          ih0 = (rem / g.OW) * g.sh - g.ph;
          iw0 = (rem % g.OW) * g.sw - g.pw;
          rbase = n_img * g.xs_n + (int64_t)ih0 * g.xs_h + (int64_t)iw0 * g.xs_w;
        }
        for (int kb = 0; kb < g.kblocks; ++kb) {
          if (!tc::mbar_wait(&empty[stage], phase ^ 1, g.err)) {
            ok = false;
            break;
          }
          uint8_t* s = smem + stage * Cfg::STAGE_BYTES;
          if (t == 0) {
            tc::mbar_arrive_expect_tx(&full[stage], SPLIT * Cfg::B_BYTES);
            uint8_t* sb = s + SPLIT * Cfg::A_BYTES;
            tc::tma_load_2d(sb, &tmW0, &full[stage], kb * BK, nt * BN);
            if (SPLIT == 2) tc::tma_load_2d(sb + Cfg::B_BYTES, &tmW1, &full[stage], kb * BK, nt * BN);
          }
          const uint32_t drow = tc::smem_u32(s) + r * 128;
#pragma unroll 4
          for (int q = 0; q < kElemPerThread; ++q) {
            const int kk = kElemPerThread * h + q;
            const int k = kb * BK + kk;
            const int hw = ktab_hw[k];
            const int ih = ih0 + (hw >> 16), iw = iw0 + (hw & 0xffff);
            const bool v = hw >= 0 && (unsigned)ih < (unsigned)g.H && (unsigned)iw < (unsigned)g.W;
            const int64_t off = v ? rbase + ktab_off[k] : 0;
            const uint32_t d = drow + (((kk >> 2) ^ (r & 7)) << 4) + ((kk & 3) << 2);
            cp_async4(d, g.x_hi + off, v ? 4u : 0u);
            if (SPLIT == 2) cp_async4(d + Cfg::A_BYTES, g.x_lo + off, v ? 4u : 0u);
          }
          cp_async_arrive_noinc(&full[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
    // Let every cp.async of this thread land before the CTA can exit.
    asm volatile("cp.async.wait_all;" ::: "memory");
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc = tc::idesc_tf32(BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;  // accumulator fills so far (tiles, or 3xTF32 chunks)
      bool ok = true;
      // 3xTF32: each chunk of kChunkKBlocks k-blocks starts a fresh
      // accumulator in the next buffer (see tc::promote_chunk32).
      const int chunk_kb = SPLIT == 2 ? tc::kChunkKBlocks : g.kblocks;
      const int chunks = SPLIT == 2 ? (g.kblocks + chunk_kb - 1) / chunk_kb : 1;
      for (int64_t t = blockIdx.x; t < g.tiles && ok; t += gridDim.x) {
       for (int ci = 0, kc = 0; ci < chunks && ok; ++ci, kc += chunk_kb, ++local) {
        const int acc = local & 1;
        const uint32_t aphase = (local >> 1) & 1;
        if (!tc::mbar_wait(&tempty[acc], aphase ^ 1, g.err)) {
          ok = false;
          break;
        }
        tc::tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        const int kend = kc + chunk_kb < g.kblocks ? kc + chunk_kb : g.kblocks;
        for (int kb = kc; kb < kend; ++kb) {
          if (!tc::mbar_wait(&full[stage], phase, g.err)) {
            ok = false;
            break;
          }
          // The A tile's cp.async writes are complete once the stage barrier
          // phase completes (cp.async.mbarrier.arrive tracks them); the
          // tcgen05 fence orders the MMAs after that wait, as in CUTLASS's
          // SM100 cp.async mainloop.
          tc::tc_fence_after();
          const uint32_t sa = tc::smem_u32(smem + stage * Cfg::STAGE_BYTES);
          const uint32_t sb = sa + SPLIT * Cfg::A_BYTES;
          const bool a_cols = g.mode == kIm2col16;
#pragma unroll
          for (int k = 0; k < BK / 8; ++k) {
            // A: 128-byte swizzled rows (advance 32 bytes per k-step), or
            // 2 KB core-matrix columns of 4 channels (two per k-step).
            const uint64_t a0 = a_cols ? tc::desc_kmajor_noswizzle(sa + k * 4096, 2048, 128)
                                       : tc::desc_kmajor_sw128(sa + k * 32);
            const uint64_t b0 = tc::desc_kmajor_sw128(sb + k * 32);
            const uint32_t accum = ((kb - kc) | k) != 0;
            if (SPLIT == 1) {
              tc::mma_tf32(d_tmem, a0, b0, idesc, accum);
            } else {
              const uint32_t sa1 = sa + Cfg::A_BYTES;
              const uint64_t a1 = a_cols ? tc::desc_kmajor_noswizzle(sa1 + k * 4096, 2048, 128)
                                         : tc::desc_kmajor_sw128(sa1 + k * 32);
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
      }
      tc::mma_commit(done);
      tc::mbar_wait(done, 0, g.err);
    }
  } else {
    // ---------------- epilogue (warps 5..12) ----------------
    // Warp w reads TMEM lanes [32 (w % 4), +32) (the hardware's lane
    // quadrant rule); the two warps of a quadrant take alternate 32-column
    // chunks.
    const int quad = warp & 3, half = (warp - kMmaWarp - 1) >> 2;
    float* stage_tile = epi + (warp - kMmaWarp - 1) * 32 * (kStageCols + 1);  // this warp's 32 x 33 tile
    const bool vec_ok = (g.Cout % 4 == 0) && ((((uintptr_t)g.out) & 15) == 0) &&
                        (!g.residual || ((((uintptr_t)g.residual) & 15) == 0));
    const bool bias_vec = g.bias && ((((uintptr_t)g.bias) & 15) == 0);
    const bool direct = vec_ok && perm_rows(g.Cout) && g.direct_epi;
    if constexpr (SPLIT == 1) {
      int local = 0;
      for (int64_t t = blockIdx.x; t < g.tiles; t += gridDim.x, ++local) {
        const int mt = (int)(t / g.n_tiles), nt = (int)(t % g.n_tiles);
        const int acc = local & 1;
        const uint32_t aphase = (local >> 1) & 1;
        if (!tc::mbar_wait(&tfull[acc], aphase, g.err)) break;
        tc::tc_fence_after();
        store_tile<BN, false>(g, tmem_base, acc * BN, nt, quad, half * kStageCols, 2 * kStageCols,
                              lane, stage_tile, vec_ok, bias_vec, LinearRows{(int64_t)mt * BM, g.M},
                              direct);
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&tempty[acc]);
      }
    } else {
    const int chunk_kb = tc::kChunkKBlocks;
    int local = 0;
    bool ok = true;
    for (int64_t t = blockIdx.x; t < g.tiles && ok; t += gridDim.x) {
      const int mt = (int)(t / g.n_tiles), nt = (int)(t % g.n_tiles);
      for (int kc = 0; kc < g.kblocks; kc += chunk_kb, ++local) {
        const int acc = local & 1;
        const uint32_t aphase = (local >> 1) & 1;
        if (!tc::mbar_wait(&tfull[acc], aphase, g.err)) {
          ok = false;
          break;
        }
        tc::tc_fence_after();
        const bool last = kc + chunk_kb >= g.kblocks;
        if (!(kc == 0 && last)) {
          // 3xTF32 chunk: fold the partial sums of this warp's column slices
          // into the running sum (columns 2 BN + c).
          const uint32_t lane_addr = tmem_base + ((uint32_t)(quad * 32) << 16);
#pragma unroll 1
          for (int c0 = half * kStageCols; c0 < BN; c0 += 2 * kStageCols) {
            if (nt * BN + c0 >= g.Cout) continue;  // warp-uniform
            tc::promote_chunk32(lane_addr, acc * BN + c0, 2 * BN + c0, kc == 0, last);
          }
          tc::tmem_st_wait();
        }
        if (last)
          store_tile<BN, false>(g, tmem_base, acc * BN, nt, quad, half * kStageCols,
                                2 * kStageCols, lane, stage_tile, vec_ok, bias_vec,
                                LinearRows{(int64_t)mt * BM, g.M}, direct);
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&tempty[acc]);
      }
    }
    }  // SPLIT == 2
  }

  tc::tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// ----------------------------------------------- paired im2col kernel ----
//
// The im2col route for C_out > 64 (ResNet stages 2-4) on CTA pairs
// (tcgen05 cta_group::2): a cluster of two CTAs computes one tile of 256
// output pixels x BN (128 or 256) channels. CTA r loads the im2col A tile of pixels
// [m0 + 128 r, +128) and rows [n0 + 128 r, +128) of the weight tile; the even
// CTA issues M = 256 MMAs that read both CTAs' operands at the same shared
// offsets and accumulate into both CTAs' TMEM (CTA r's 128 lanes hold its
// pixels x all 256 channels). Per k-block each SM receives 16 KB of A and
// 16 KB of B instead of 16 + 32 KB, which is what bounds the single-CTA
// kernel's N = 256 MMAs (TMA delivers ~52 B/clk of im2col rows and ~80 of
// tiled rows per SM; the MMAs consume a k-block in 512 cycles).
//
// Barriers: the stage barriers full[s] of the even CTA count both CTAs' TMA
// bytes (the loads name it through .cta_group::2); the even CTA's commits
// arrive on empty[s], tfull[a] and done in both CTAs; every epilogue warp of
// both CTAs arrives on the even CTA's tempty[a] (16 arrivals). Cluster
// barriers after set-up and before the pair's TMEM is freed; the odd CTA
// waits for the final commit before it leaves. No TMA load uses cluster
// multicast.
//
// Stream-K (g.sk_q > 0, chosen by the host when whole tiles would leave the
// last wave of pairs less than 90% full): after its whole tiles each cluster
// takes an equal share of the remaining tiles' k-block iterations, walking
// its share from its last tile to its first. A share that begins a tile
// (or sits inside one) stops before the tile's last k-block: the cluster
// writes those partial sums to its slot first thing and counts its 16
// epilogue warps in on the slot's counter. The share that ends a tile does
// that tile's epilogue last thing: it waits for the slots of the clusters
// before it, adds them to its accumulator in cluster order (so the result is
// the same on every run) and counts itself in; the last of the 32 arrivals
// puts the counter back to zero for the next launch. A cluster only ever
// waits for lower-numbered clusters, whose partial units come first.
struct PairUnit {
  int64_t tile;
  int kb0, kb1;  // k-blocks [kb0, kb1) of the tile
};
// SK = false: whole tiles only, every clusters-th tile from the cluster's own.
template <bool SK>
struct PairSchedule {
  int64_t lo, hi;  // this cluster's stream-K share [lo, hi) (iteration = tile * KB + kb)
  __device__ PairSchedule(const ConvArgs& g) : lo(0), hi(0) {
    if (SK) {
      const int64_t c = cluster();
      lo = g.sk_dp_tiles * g.kblocks + c * g.sk_q + (c < g.sk_r ? c : g.sk_r);
      hi = lo + g.sk_q + (c < g.sk_r ? 1 : 0);
    }
  }
  // The cluster (CTA pair) and the number of clusters of this launch.
  static __device__ int cluster() { return (int)(blockIdx.x >> 1); }
  static __device__ int clusters() { return (int)(gridDim.x >> 1); }
  static __device__ int64_t n_dp(const ConvArgs& g) {
    const int64_t dp_end = SK ? g.sk_dp_tiles : g.tiles;
    return cluster() < dp_end ? (dp_end - 1 - cluster()) / clusters() + 1 : 0;
  }
  __device__ int64_t count(const ConvArgs& g) const {
    return n_dp(g) + (SK && hi > lo ? (hi - 1) / g.kblocks - lo / g.kblocks + 1 : 0);
  }
  __device__ PairUnit unit(const ConvArgs& g, int64_t u) const {
    const int KB = g.kblocks;
    if (!SK) return {cluster() + u * clusters(), 0, KB};
    const int64_t nd = n_dp(g);
    if (u < nd) return {cluster() + u * clusters(), 0, KB};
    const int64_t t_hi = (hi - 1) / KB, t = t_hi - (u - nd);
    return {t, t == lo / KB ? (int)(lo - t * KB) : 0, t == t_hi ? (int)(hi - t * KB) : KB};
  }
  // The cluster whose share holds iteration `it` (stream-K tiles only).
  static __device__ int64_t owner(const ConvArgs& g, int64_t it) {
    const int64_t rel = it - g.sk_dp_tiles * g.kblocks, split = g.sk_r * (g.sk_q + 1);
    return rel < split ? rel / (g.sk_q + 1) : g.sk_r + (rel - split) / g.sk_q;
  }
};

constexpr unsigned kSkWarps = 2 * kEpilogueWarps;  // arrivals per side of a slot

// A slot holds, per CTA of the pair, 128 rows x BN columns in 16-column
// chunks of one warp (32 rows x 16 columns, 2 KB): chunk (quad, cc) at
// float offset (quad * BN / 16 + cc) * 512, and inside it lane l's four
// float4 at (j * 32 + l) * 4, so each warp-wide access covers 512
// contiguous bytes. The warps of half h take the 32-column groups h, h + 2,
// ... (chunks 4 i + 2 h and 4 i + 2 h + 1): the columns store_tile has the
// same warp write out, so a warp's fixed-up sums are its own to read.
template <int BN>
__device__ __forceinline__ float4* sk_chunk(float* slot, int quad, int cc) {
  return reinterpret_cast<float4*>(slot + (size_t)(quad * (BN / 16) + cc) * 512);
}

// Partial sums of this warp's rows and chunks -> the slot (TMEM address
// `acc` = this warp's lane quadrant at the accumulator's first column).
template <int BN>
__device__ __forceinline__ void sk_save(float* slot, uint32_t acc, int quad, int half, int lane) {
#pragma unroll 1
  for (int cc = 2 * half; cc < BN / 16; cc += 1 + 2 * (cc & 1)) {
    uint32_t r[16];
    tc::tmem_ld16(acc + cc * 16, r);
    tc::tmem_ld_wait();
    float4* dst = sk_chunk<BN>(slot, quad, cc);
#pragma unroll
    for (int j = 0; j < 4; ++j)
      __stcg(dst + j * 32 + lane, make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                              __uint_as_float(r[4 * j + 2]),
                                              __uint_as_float(r[4 * j + 3])));
  }
}

// Bounded wait (every lane) until *count reaches `want`; acquire ordering.
__device__ __forceinline__ bool sk_wait(const unsigned* count, unsigned want, int* err) {
  const uint64_t t0 = tc::global_ns();
  for (uint32_t i = 0; i < tc::kWaitLimit; ++i) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(count) : "memory");
    if (v >= want) return true;
    if (tc::global_ns() - t0 > tc::kWaitNs) break;
    __nanosleep(200);
  }
  if (err) atomicExch(err, 5 /* NNC_CUDA_ERR_DEVICE_TIMEOUT */);
  return false;
}

// Adds the slots of clusters [first, last) to this warp's accumulator
// chunks, in cluster order, once each slot's writers are all in; then
// counts this warp in on each slot (the last arrival zeroes the counter).
// A chunk's TMEM load and its first partial-sum loads are in flight
// together.
template <int BN>
__device__ __forceinline__ void sk_fixup(const ConvArgs& g, int64_t first, int64_t last,
                                         uint32_t rank, uint32_t acc, int quad, int half,
                                         int lane) {
  const size_t slot_floats = (size_t)2 * BM * BN;
  bool ok = true;
  for (int64_t s = first; s < last; ++s) ok = sk_wait(&g.sk_count[s], kSkWarps, g.err) && ok;
  ok = __all_sync(0xffffffffu, ok) && first < last;
#pragma unroll 1
  for (int cc = 2 * half; cc < BN / 16; cc += 1 + 2 * (cc & 1)) {
    uint32_t r[16];
    tc::tmem_ld16(acc + cc * 16, r);
    for (int64_t s = first; s < last && ok; ++s) {
      const float4* src = sk_chunk<BN>(g.sk_part + s * slot_floats + rank * (BM * BN), quad, cc);
      float4 p[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) p[j] = __ldcg(src + j * 32 + lane);
      if (s == first) tc::tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        r[4 * j] = __float_as_uint(__fadd_rn(__uint_as_float(r[4 * j]), p[j].x));
        r[4 * j + 1] = __float_as_uint(__fadd_rn(__uint_as_float(r[4 * j + 1]), p[j].y));
        r[4 * j + 2] = __float_as_uint(__fadd_rn(__uint_as_float(r[4 * j + 2]), p[j].z));
        r[4 * j + 3] = __float_as_uint(__fadd_rn(__uint_as_float(r[4 * j + 3]), p[j].w));
      }
    }
    if (!ok) tc::tmem_ld_wait();
    tc::tmem_st16(acc + cc * 16, r);
  }
  tc::tmem_st_wait();
  __syncwarp();
  if (lane == 0 && ok)
    for (int64_t s = first; s < last; ++s)
      if (atomicAdd(&g.sk_count[s], 1u) == 2 * kSkWarps - 1) atomicExch(&g.sk_count[s], 0u);
}

template <int BN_, int STAGES>
struct ConvPairCfg {
  static constexpr int BN = BN_;        // MMA N (128 or 256); each CTA holds BN / 2 weight rows
  static constexpr uint32_t A_BYTES = BM * BK * 4;             // 16 KB
  static constexpr uint32_t B_BYTES = (BN / 2) * BK * 4;       // 8 or 16 KB
  static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr uint32_t TMEM_COLS = 2 * BN;                // double-buffered accumulator
  static constexpr uint32_t EPI_OFF = STAGES * STAGE_BYTES;
  static constexpr uint32_t BAR_OFF = EPI_OFF + kEpiBytes;
  static constexpr size_t SMEM = (size_t)BAR_OFF + 256 + 1024;
};

// 10 warps: warp 0 produces (one thread), warp 1 issues (even CTA), warps
// 2..9 drain TMEM; 3 warps per SM sub-partition at most leave 168 registers
// per thread, room for the direct epilogue.
constexpr int kPairMmaWarp = 1, kPairThreads = 32 * (2 + kEpilogueWarps);
template <int BN_, int STAGES, bool SK>
__global__ void __launch_bounds__(kPairThreads, 1)
    conv_tc2_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                    const ConvArgs g) {
  using Cfg = ConvPairCfg<BN_, STAGES>;
  constexpr int BN = Cfg::BN;
  extern __shared__ uint8_t smem_raw[];
  pdl_trigger();
  uint8_t* smem = align1024(smem_raw);
  float* epi = reinterpret_cast<float*>(smem + Cfg::EPI_OFF);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::BAR_OFF);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* done = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = tc::cluster_ctarank();  // 0: issues the MMAs

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(&full[s], 1);   // even CTA: its expect_tx arrival (+ both CTAs' bytes)
      tc::mbar_init(&empty[s], 1);  // one pair commit
    }
    for (int a = 0; a < 2; ++a) {
      tc::mbar_init(&tfull[a], 1);
      tc::mbar_init(&tempty[a], 2 * kEpilogueWarps);  // even CTA: both CTAs' epilogue warps
    }
    tc::mbar_init(done, 1);
    tc::fence_barrier_init();
    tc::prefetch_tmap(&tmW);
    tc::prefetch_tmap(&tmX);
  }
  if (warp == kPairMmaWarp) {
    tc::tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
    tc::tmem_relinquish_pair();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::cluster_sync();  // both CTAs' barriers initialised, TMEM allocated
  tc::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // the previous kernel's outputs are complete from here on

  if (warp < kPairMmaWarp) {
    // ---------------- producer (one thread per CTA): A half, B half ----------------
    if (threadIdx.x == 0) {
      const int64_t OHW = (int64_t)g.OH * g.OW;
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      const PairSchedule<SK> sch(g);
      for (int64_t u = 0; u < sch.count(g) && ok; ++u) {
        const PairUnit pu = sch.unit(g, u);
        const int64_t mt = pu.tile / g.n_tiles;
        const int nt = (int)(pu.tile % g.n_tiles);
        // This CTA's first pixel; a half past the last pixel loads the
        // pair's first half again (valid coordinates; its rows are masked).
        int64_t m0 = mt * (2 * BM) + (int64_t)rank * BM;
        if (m0 >= g.M) m0 = mt * (2 * BM);
        const int n0 = (int)(m0 / OHW);
        const int rem = (int)(m0 - (int64_t)n0 * OHW);
        const int w0 = (rem % g.OW) * g.sw - g.pw, h0 = (rem / g.OW) * g.sh - g.ph;
        for (int kb = pu.kb0; kb < pu.kb1; ++kb) {
          if (!tc::mbar_wait(&empty[stage], phase ^ 1, g.err)) {
            ok = false;
            break;
          }
          uint8_t* s = smem + stage * Cfg::STAGE_BYTES;
          if (rank == 0) tc::mbar_arrive_expect_tx(&full[stage], 2 * Cfg::STAGE_BYTES);
          const uint32_t bar = tc::mapa(tc::smem_u32(&full[stage]), 0);
          tc::tma_load_2d_pair(s + Cfg::A_BYTES, &tmW, bar, kb * BK, nt * BN + (int)rank * (BN / 2));
          const int k0 = kb * BK, tap = k0 / g.C4, c0 = k0 - tap * g.C4;
          const uint16_t kh = (uint16_t)(tap / g.KW), kw = (uint16_t)(tap % g.KW);
          tc::tma_load_im2col_4d_pair(s, &tmX, bar, c0, w0, h0, n0, kw, kh);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // The even CTA lets the last issued loads of both CTAs land before it
      // can leave (the odd CTA's loads count on these barriers too).
      if (ok && rank == 0) {
        for (int q = 0; q < STAGES; ++q) {
          if (stage == 0) {
            stage = STAGES;
            phase ^= 1;
          }
          --stage;
          tc::mbar_wait(&full[stage], phase, g.err);
        }
      }
    }
  } else if (warp == kPairMmaWarp) {
    if (rank == 0 && lane == 0) {
      // ---------------- MMA issuer (even CTA) ----------------
      constexpr uint32_t idesc = tc::idesc_tf32(2 * BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      const PairSchedule<SK> sch(g);
      for (int64_t u = 0; u < sch.count(g) && ok; ++u, ++local) {
        const PairUnit pu = sch.unit(g, u);
        const int acc = local & 1;
        const uint32_t aphase = (local >> 1) & 1;
        if (!tc::mbar_wait(&tempty[acc], aphase ^ 1, g.err)) break;
        tc::tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = pu.kb0; kb < pu.kb1; ++kb) {
          if (!tc::mbar_wait(&full[stage], phase, g.err)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t sa = tc::smem_u32(smem + stage * Cfg::STAGE_BYTES);
          const uint32_t sb = sa + Cfg::A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 8; ++k)
            tc::mma_tf32_pair(d_tmem, tc::desc_kmajor_sw128(sa + k * 32),
                              tc::desc_kmajor_sw128(sb + k * 32), idesc,
                              ((kb - pu.kb0) | k) != 0);
          tc::mma_commit_pair_both(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        tc::mma_commit_pair_both(&tfull[acc]);
      }
      tc::mma_commit_pair_both(done);
      tc::mbar_wait(done, 0, g.err);
    }
  } else {
    // ---------------- epilogue (warps 2..9 of both CTAs) ----------------
    const int quad = warp & 3, half = (warp - kPairMmaWarp - 1) >> 2;
    float* stage_tile = epi + (warp - kPairMmaWarp - 1) * 32 * (kStageCols + 1);
    const bool vec_ok = (g.Cout % 4 == 0) && ((((uintptr_t)g.out) & 15) == 0) &&
                        (!g.residual || ((((uintptr_t)g.residual) & 15) == 0));
    const bool bias_vec = g.bias && ((((uintptr_t)g.bias) & 15) == 0);
    const bool direct = vec_ok && perm_rows(g.Cout) && g.direct_epi;
    const uint32_t tempty0 = tc::mapa(tc::smem_u32(&tempty[0]), 0);
    int local = 0;
    const PairSchedule<SK> sch(g);
    for (int64_t u = 0; u < sch.count(g); ++u, ++local) {
      const PairUnit pu = sch.unit(g, u);
      const int64_t mt = pu.tile / g.n_tiles;
      const int nt = (int)(pu.tile % g.n_tiles);
      const int acc = local & 1;
      const uint32_t aphase = (local >> 1) & 1;
      if (!tc::mbar_wait(&tfull[acc], aphase, g.err)) break;
      tc::tc_fence_after();
      const uint32_t acc_addr = tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BN;
      if (SK && pu.kb1 < g.kblocks) {
        // Partial unit: sums to this cluster's slot, buffer back to the
        // issuer, then the slot's writers count in (stores visible first).
        const int me = PairSchedule<SK>::cluster();
        sk_save<BN>(g.sk_part + (size_t)me * (2 * BM * BN) + rank * (BM * BN), acc_addr, quad, half,
                    lane);
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive_cluster(tempty0 + acc * (uint32_t)sizeof(uint64_t));
        __threadfence();
        __syncwarp();
        if (lane == 0) atomicAdd(&g.sk_count[me], 1u);
        continue;
      }
      if (SK && pu.kb0 > 0)
        sk_fixup<BN>(g, PairSchedule<SK>::owner(g, pu.tile * g.kblocks), PairSchedule<SK>::cluster(),
                     rank, acc_addr, quad, half, lane);
      store_tile<BN, true>(g, tmem_base, acc * BN, nt, quad, half * kStageCols, 2 * kStageCols,
                           lane, stage_tile, vec_ok, bias_vec,
                           LinearRows{mt * (2 * BM) + (int64_t)rank * BM, g.M}, direct);
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive_cluster(tempty0 + acc * (uint32_t)sizeof(uint64_t));
    }
    // The odd CTA leaves only after the even CTA's last commit has arrived
    // here (its barriers receive the pair's commits).
    if (rank == 1 && warp == kPairMmaWarp + 1) tc::mbar_wait_warp(done, 0, g.err);
  }

  tc::tc_fence_before();
  __syncthreads();
  tc::cluster_sync();  // no CTA frees the pair's TMEM or leaves while the other works
  if (warp == kPairMmaWarp) {
    tc::tc_fence_after();
    tc::tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
  }
}

// --------------------------------------------------------- halo kernel ----
//
// Stride-1 convolutions (and 1 x 1 windows with stride 2) over an NHWC input
// whose stored channel count C4 is a multiple of the channel block. A tile is
// an 8-wide x 32-tall block of one image's output pixels, split into an upper
// and a lower 8 x 16 block (one 128-row accumulator each, row r = 8 y + x),
// times BN <= 128 output channels.
//
// Per 32-channel block one TMA load brings the tile's input window,
// (32 + KH - 1) x (8 + KW - 1) pixels of 128 bytes in the 128-byte swizzle
// layout, zero-filled outside the image (the padding). Every tap's A operand
// is a descriptor into that window: tap (kh, kw) of the upper block starts at
// window row kh (8 + KW - 1) + kw (the lower block 16 window rows further),
// and its 8-row groups (one output row each) lie (8 + KW - 1) rows apart: the
// swizzle follows absolute shared addresses, so any 128-byte row may start a
// group. Only BN x 32 weight tiles stream per tap, G taps per ring stage, and
// both blocks read the same stage.
//
// Issue rate: an mbarrier wait costs ~100 cycles even when the phase has
// completed, and the tensor pipe runs only ~2 MMAs ahead of one issuing
// thread, so a single issuer idles an N = 64 or 128 pipe at every wait. Two
// MMA warps (one per block, separate accumulators) keep it busy: while one
// waits the other issues, and measured together they reach the pipe's full
// rate. Each loop runs on its whole warp with one elected lane issuing, and
// descriptors advance by addition only.
//
// 352 threads: warp 0 lane 0 issues the TMA loads; warps 1 and 2 (upper,
// lower block) issue the MMAs, warp 1 owning TMEM; warps 3..6 drain the upper
// accumulators and warps 7..10 the lower ones (shared epilogue, store_tile).
//
// POOL: the conv result (bias, ReLU) is max-pooled in the epilogue and only
// the pooled tensor is written. A CTA then takes whole images and walks their
// tiles in raster order, keeping in shared memory the previous tile's last
// column and the previous tile row's last conv row, so every pooled window
// (stride 2, at most one row/column before its centre and one after) is
// complete in the tile that holds its centre: no atomics, no second pass.
constexpr int kHaloTW = 8, kHaloTH = 16;  // one accumulator block
constexpr int kHaloMaxK = 4;               // largest KH and KW
constexpr int kHaloSlots = 2;
constexpr int kHaloThreads = 32 * (3 + kEpilogueWarps);
constexpr int kGatherThreads = 128;  // GATHER: four window-building warps after the epilogue
constexpr int kPoolMaxOW = 128;  // widest conv output the pooled epilogue carries a row of
// POOL shared buffers. A thread's 8 values of a 32-channel chunk travel as
// two float4 runs u = 0, 1 (values 4 u .. 4 u + 3), every run at a
// 16-byte slot so each warp access is one conflict-free 128-byte wavefront
// per 8 threads: the exchange of each warp's last conv row with the warp
// below it ([chunk parity][u][8 row groups][32 threads] float4), the row
// carry ([kPoolMaxOW columns] x BN values at a BN + 16 stride, value order
// [chunk][u][thread & 3][4]) and the column carry ([8 row groups][2 centre
// rows][chunk][u][thread & 3] float4).
constexpr uint32_t kPoolXchgFloats = 2 * 2 * 8 * 32 * 4;

// CB: channels per window row, 32 (128-byte rows, 128-byte swizzle) or 16
// (64-byte rows, 64-byte swizzle: the space-to-depth stem's 12 channels).
// STAGED = false: the instance serves only calls whose epilogue takes the
// direct path (no shared staging tile; the space goes to the weight ring).
template <int BN, int G, int STAGES, int CB, bool POOL = false, bool STAGED = true,
          bool PAIR = false, bool GATHER = false>
struct HaloCfg {
  static constexpr int SLOTS = kHaloSlots;  // window slots
  static constexpr int ROW = CB * 4;                    // bytes per window row
  static constexpr uint32_t SLOT_BYTES = (2 * kHaloTH + kHaloMaxK - 1) *
                                             (kHaloTW + kHaloMaxK - 1) * ROW / 1024 * 1024 + 1024;
  // One tap's weight tile (PAIR: this CTA's half of the BN rows).
  static constexpr uint32_t B_BYTES = (PAIR ? BN / 2 : BN) * CB * 4;
  static constexpr uint32_t STAGE_BYTES = G * B_BYTES;  // G taps per ring stage
  static constexpr uint32_t HALO_OFF = STAGES * STAGE_BYTES;
  static constexpr uint32_t EPI_OFF = HALO_OFF + SLOTS * SLOT_BYTES;
  static constexpr uint32_t EPI_BYTES = POOL ? kPoolXchgFloats * 4 : (STAGED ? kEpiBytes : 0);
  static constexpr uint32_t CARRY_OFF = EPI_OFF + EPI_BYTES;
  static constexpr int ROW_CARRY_STRIDE = BN + 16;
  static constexpr uint32_t CARRY_BYTES =
      POOL ? (uint32_t)(kPoolMaxOW * ROW_CARRY_STRIDE + 16 * BN) * 4 : 0;
  static constexpr uint32_t BAR_OFF = CARRY_OFF + CARRY_BYTES;
  static constexpr uint32_t TMEM_COLS = 4 * BN;  // {upper, lower} x double buffer
  static constexpr size_t SMEM = (size_t)BAR_OFF + 256 + 1024;
};

__device__ __forceinline__ void epi_bar_sync() {
  asm volatile("bar.sync 1, 256;" ::: "memory");  // the 8 epilogue warps
}

// POOL epilogue of one tile, run by all 8 epilogue warps. Warp (blk, quad)
// holds tile rows 4 G .. 4 G + 3, G = 4 blk + quad, as TMEM lanes 32 quad +
// 8 yy + x. Per 32-channel chunk each warp reads its lanes with two 16x256b
// loads, so thread t holds column x = t >> 2 of all four rows at TMEM columns
// 8 q + 2 (t & 3) + {0, 1}, q = 0..3 (value j = 2 q + h; channel perm_col of
// the column when C_out is a multiple of 32, which makes values 4 u .. 4 u + 3
// channels 16 u + 4 (t & 3) + {0..3}):
//   vertical   centre rows yy = 0, 2 take rows yy - 1 .. yy + 1 from
//              registers; row -1 is the last row of the warp above, passed
//              through shared memory (the row carry for G = 0);
//   horizontal centre columns x = 0, 2, 4, 6 take x +- 1 from threads t +- 4
//              by shuffle; column -1 is the previous tile's column 7 (the
//              column carry).
// Shared memory and shuffles are the scarce resource here (the MMAs of the
// next tile hold the shared-memory port), so every shared access moves a
// float4 and the buffers are laid out conflict-free.
// ReLU results are >= 0 and never NaN, so the maximum is order-free, and a
// zero stands for window positions outside the conv result (a window always
// holds its centre, so none is empty): the reference's first-then-strictly-
// greater scan gives the same values. `parity` counts chunks (the exchange
// buffer alternates).
__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ void st4(float* p, const float* v) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
}
template <int BN>
__device__ __forceinline__ void pool_tile(const ConvArgs& g, uint32_t tmem_base, int acc, int blk,
                                          int quad, int lane, float* xchg, float* row_carry,
                                          float* col_carry, uint32_t& parity, int n, int y0,
                                          int x0) {
  constexpr int RS = BN + 16;  // row carry stride (floats per column)
  const int G = 4 * blk + quad;
  const int x = lane >> 2, cp = lane & 3;
  const bool up = g.pph == 1, down = g.pkh - g.pph == 2;
  const bool left = g.ppw == 1, right = g.pkw - g.ppw == 2;
  const bool col_in = x0 + x < g.OW;
  bool row_in[4];
#pragma unroll
  for (int yy = 0; yy < 4; ++yy) row_in[yy] = col_in && y0 + 4 * G + yy < g.OH;
  const bool centre_x = (x & 1) == 0 && (x0 + x) / 2 < g.PW;
  const int py0 = (y0 + 4 * G) / 2;  // pooled row of centre row yy = 0 (yy = 2: + 1)
  const bool st0 = centre_x && py0 < g.PH, st2 = centre_x && py0 + 1 < g.PH;
  float* const out0 = g.out + (((int64_t)n * g.PH + py0) * g.PW + (x0 + x) / 2) * g.Cout;
  float* const out2 = out0 + (int64_t)g.PW * g.Cout;
  const bool perm = perm_rows(g.Cout);
  const bool pair_ok = (g.Cout & 1) == 0 && ((((uintptr_t)g.out) & 7) == 0);
  const bool quad_ok = perm && ((((uintptr_t)g.out) & 15) == 0);
  int chunk = 0;
  for (int c0 = 0; c0 < BN && c0 < g.Cout; c0 += 32, ++chunk) {
    const uint32_t taddr =
        tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * 2 + blk) * BN + c0;
    uint32_t ra[16], rb[16];
    __syncwarp();  // tcgen05.ld is .sync.aligned: the warp must be converged
    tc::tmem_ld_16x256b_x4(taddr, ra);               // rows yy = 0, 1
    tc::tmem_ld_16x256b_x4(taddr + (16u << 16), rb);  // rows yy = 2, 3
    // Value j = 2 q + h is TMEM column 8 q + 2 cp + h of the chunk.
    float bj[8];
    if (perm && g.bias && ((((uintptr_t)g.bias) & 15) == 0)) {
      const float4 b0 = __ldg(reinterpret_cast<const float4*>(g.bias + c0 + 4 * cp));
      const float4 b1 = __ldg(reinterpret_cast<const float4*>(g.bias + c0 + 16 + 4 * cp));
      bj[0] = b0.x; bj[1] = b0.y; bj[2] = b0.z; bj[3] = b0.w;
      bj[4] = b1.x; bj[5] = b1.y; bj[6] = b1.z; bj[7] = b1.w;
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int col = 8 * (j >> 1) + 2 * cp + (j & 1);
        const int ch = c0 + (perm ? perm_col(col) : col);
        bj[j] = (g.bias && ch < g.Cout) ? __ldg(g.bias + ch) : 0.0f;
      }
    }
    // Row -1 of group 0 is the row carry (zeros at the image's top edge);
    // read before the barrier, after which group 7 overwrites it.
    float above[8];
    float* const rc = row_carry + (x0 + x) * RS + chunk * 32 + 4 * cp;  // + 16 u
    if (G == 0) {
      const bool live = up && y0 > 0 && col_in;
      const float4 a0 = live ? ld4(rc) : make_float4(0.f, 0.f, 0.f, 0.f);
      const float4 a1 = live ? ld4(rc + 16) : make_float4(0.f, 0.f, 0.f, 0.f);
      above[0] = a0.x; above[1] = a0.y; above[2] = a0.z; above[3] = a0.w;
      above[4] = a1.x; above[5] = a1.y; above[6] = a1.z; above[7] = a1.w;
    }
    tc::tmem_ld_wait();
    float v[4][8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int q = j >> 1, h = j & 1;
      const float a0 = __fadd_rn(__uint_as_float(ra[4 * q + h]), bj[j]);
      const float a1 = __fadd_rn(__uint_as_float(ra[4 * q + 2 + h]), bj[j]);
      const float a2 = __fadd_rn(__uint_as_float(rb[4 * q + h]), bj[j]);
      const float a3 = __fadd_rn(__uint_as_float(rb[4 * q + 2 + h]), bj[j]);
      v[0][j] = (row_in[0] && a0 > 0.0f) ? a0 : 0.0f;
      v[1][j] = (row_in[1] && a1 > 0.0f) ? a1 : 0.0f;
      v[2][j] = (row_in[2] && a2 > 0.0f) ? a2 : 0.0f;
      v[3][j] = (row_in[3] && a3 > 0.0f) ? a3 : 0.0f;
    }
    // Exchange slot of group G's last row: [parity][u][G + 1][lane] float4.
    float* const xb = xchg + (parity & 1) * (2 * 8 * 32 * 4);
    if (G < 7) {
      st4(xb + ((0 * 8 + G + 1) * 32 + lane) * 4, &v[3][0]);
      st4(xb + ((1 * 8 + G + 1) * 32 + lane) * 4, &v[3][4]);
    }
    epi_bar_sync();
    if (G > 0) {
      const float4 a0 = ld4(xb + ((0 * 8 + G) * 32 + lane) * 4);
      const float4 a1 = ld4(xb + ((1 * 8 + G) * 32 + lane) * 4);
      above[0] = a0.x; above[1] = a0.y; above[2] = a0.z; above[3] = a0.w;
      above[4] = a1.x; above[5] = a1.y; above[6] = a1.z; above[7] = a1.w;
    }
    // This tile's last row replaces the row carry for the tile row below
    // (group 0 read the old one before the barrier).
    if (G == 7 && col_in) {
      st4(rc, &v[3][0]);
      st4(rc + 16, &v[3][4]);
    }
    // Vertical maxima of the two centre rows.
    float m0[8], m2[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float a = v[0][j], b = v[2][j];
      if (up) {
        a = fmaxf(a, above[j]);
        b = fmaxf(b, v[1][j]);
      }
      if (down) {
        a = fmaxf(a, v[1][j]);
        b = fmaxf(b, v[3][j]);
      }
      m0[j] = a;
      m2[j] = b;
    }
    // Horizontal: columns x - 1 and x + 1 are threads t - 4 and t + 4;
    // column -1 is the previous tile's column 7 (zeros at the left edge).
    float o0[8], o2[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float l0 = __shfl_up_sync(0xffffffffu, m0[j], 4);
      const float l2 = __shfl_up_sync(0xffffffffu, m2[j], 4);
      const float r0 = __shfl_down_sync(0xffffffffu, m0[j], 4);
      const float r2 = __shfl_down_sync(0xffffffffu, m2[j], 4);
      float a = m0[j], b = m2[j];
      if (left && x > 0) {
        a = fmaxf(a, l0);
        b = fmaxf(b, l2);
      }
      if (right) {
        a = fmaxf(a, r0);
        b = fmaxf(b, r2);
      }
      o0[j] = a;
      o2[j] = b;
    }
    // Column carry slot of (G, centre row, chunk, u, cp): one float4.
    float* const cc = col_carry + (((G * 2) * (BN / 32) + chunk) * 2 * 4 + cp) * 4;
    constexpr int kRowStep = (BN / 32) * 2 * 4 * 4;  // centre row yy = 2
    if (left && x == 0 && x0 > 0) {
      const float4 p0 = ld4(cc), p1 = ld4(cc + 16);
      const float4 q0 = ld4(cc + kRowStep), q1 = ld4(cc + kRowStep + 16);
      o0[0] = fmaxf(o0[0], p0.x); o0[1] = fmaxf(o0[1], p0.y);
      o0[2] = fmaxf(o0[2], p0.z); o0[3] = fmaxf(o0[3], p0.w);
      o0[4] = fmaxf(o0[4], p1.x); o0[5] = fmaxf(o0[5], p1.y);
      o0[6] = fmaxf(o0[6], p1.z); o0[7] = fmaxf(o0[7], p1.w);
      o2[0] = fmaxf(o2[0], q0.x); o2[1] = fmaxf(o2[1], q0.y);
      o2[2] = fmaxf(o2[2], q0.z); o2[3] = fmaxf(o2[3], q0.w);
      o2[4] = fmaxf(o2[4], q1.x); o2[5] = fmaxf(o2[5], q1.y);
      o2[6] = fmaxf(o2[6], q1.z); o2[7] = fmaxf(o2[7], q1.w);
    }
    __syncwarp();  // column 0's carry reads precede column 7's writes
    if (x == 7) {
      st4(cc, &m0[0]);
      st4(cc + 16, &m0[4]);
      st4(cc + kRowStep, &m2[0]);
      st4(cc + kRowStep + 16, &m2[4]);
    }
    // Pooled outputs: centre columns of centre rows. Permuted channels give
    // this thread c0 + 16 u + 4 cp + {0..3} (values 4 u .. 4 u + 3): 16-byte
    // stores; otherwise channel pairs.
    if (quad_ok) {
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int ch = c0 + 16 * u + 4 * cp;
        if (st0) st4(out0 + ch, &o0[4 * u]);
        if (st2) st4(out2 + ch, &o2[4 * u]);
      }
      ++parity;
      continue;
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int ch = c0 + (perm ? perm_col(8 * q + 2 * cp) : 8 * q + 2 * cp);
      if (ch >= g.Cout) continue;
      const bool pair = pair_ok && ch + 1 < g.Cout;
      if (st0) {
        if (pair) {
          *reinterpret_cast<float2*>(out0 + ch) = make_float2(o0[2 * q], o0[2 * q + 1]);
        } else {
          out0[ch] = o0[2 * q];
          if (ch + 1 < g.Cout) out0[ch + 1] = o0[2 * q + 1];
        }
      }
      if (st2) {
        if (pair) {
          *reinterpret_cast<float2*>(out2 + ch) = make_float2(o2[2 * q], o2[2 * q + 1]);
        } else {
          out2[ch] = o2[2 * q];
          if (ch + 1 < g.Cout) out2[ch + 1] = o2[2 * q + 1];
        }
      }
    }
    ++parity;
  }
}

// The k-th tile a CTA processes, or -1 past its last: every gridDim-th tile,
// or (POOL, one channel tile) every gridDim-th image with its tiles in
// raster order. PAIR (not with POOL): the two CTAs of a cluster take
// neighbouring tiles of one channel tile in lockstep, CTA r the r-th; a CTA
// whose neighbour is past the end gets the pair's first tile again with
// `valid` false (its MMA rows are computed and not stored), so both run out
// at the same k.
struct HaloUnit {
  int64_t tile;
  bool valid;
};
template <bool POOL, bool PAIR>
__device__ __forceinline__ HaloUnit halo_unit(const ConvArgs& g, int64_t k, uint32_t rank) {
  const int64_t per = (int64_t)g.tiles_x * g.tiles_y;
  if (!PAIR) {
    if (!POOL) {
      const int64_t t = blockIdx.x + k * gridDim.x;
      return {t < g.tiles ? t : -1, true};
    }
    const int64_t img = blockIdx.x + (k / per) * gridDim.x;
    return {img < g.N ? img * per + k % per : -1, true};
  }
  static_assert(!(POOL && PAIR), "the pooled epilogue runs on single CTAs");
  const int64_t cluster = blockIdx.x >> 1, clusters = gridDim.x >> 1;
  const int64_t pt = cluster + k * clusters;
  if (pt >= (int64_t)((g.m_tiles + 1) >> 1) * g.n_tiles) return {-1, false};
  const int64_t mt0 = 2 * (pt / g.n_tiles), mt = mt0 + rank;
  const bool valid = mt < g.m_tiles;
  return {(valid ? mt : mt0) * g.n_tiles + pt % g.n_tiles, valid};
}

// GATHER (single CTAs, CB = 16, a 3-channel source): instead of TMA window
// loads, four more warps build each tile's space-to-depth window from the
// original input: window row r = (wy, wx) is s2d pixel (y0 - ph + wy,
// x0 - pw + wx), whose channel 3 q + c (q = 2 dy + dx) is source channel c
// at (2 i + dy, 2 j + dx), zero outside the image, channels 12..15 zero. A
// row's four 16-byte chunks go where the 64-byte swizzle puts them (chunk j
// of row r at j ^ ((r >> 1) & 3): the slot is 1024-byte aligned and rows
// are 64 bytes), then a proxy fence makes the generic stores visible to
// the tensor core's reads before the warp arrives on the window barrier.
// This replaces a separate space-to-depth pass and its round trip through
// HBM.
template <int BN, int G, int STAGES, int CB, bool POOL, bool STAGED, bool PAIR, bool GATHER>
__global__ void __launch_bounds__(kHaloThreads + (GATHER ? kGatherThreads : 0), 1)
    conv_halo_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                     const ConvArgs g) {
  static_assert(!GATHER || (CB == 16 && !PAIR), "window gathering: 16-channel blocks, single CTAs");
  using Cfg = HaloCfg<BN, G, STAGES, CB, POOL, STAGED, PAIR, GATHER>;
  constexpr int kSlots = Cfg::SLOTS;
  extern __shared__ uint8_t smem_raw[];
  pdl_trigger();
  uint8_t* smem = align1024(smem_raw);
  uint8_t* halo = smem + Cfg::HALO_OFF;
  float* epi = reinterpret_cast<float*>(smem + Cfg::EPI_OFF);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::BAR_OFF);
  uint64_t* empty = full + STAGES;
  uint64_t* hfull = empty + STAGES;
  uint64_t* hempty = hfull + kSlots;
  uint64_t* tfull = hempty + kSlots;  // [acc][block]
  uint64_t* tempty = tfull + 4;           // [acc][block]
  uint64_t* done = tempty + 4;            // [block]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // PAIR: this CTA's rank in the cluster; rank 0 issues the MMAs of both.
  const uint32_t rank = PAIR ? tc::cluster_ctarank() : 0;
  const int hw = kHaloTW + g.KW - 1, hh = 2 * kHaloTH + g.KH - 1;  // window extent in pixels
  const int taps = g.KH * g.KW, cblocks = g.C4 / CB;
  const int per_img = g.tiles_x * g.tiles_y;
  // Resident weights: when one channel tile and one channel block cover the
  // call and all the tap groups fit the ring (the space-to-depth stem's 16
  // taps x 64 channels: 64 KB), the weights are loaded once per CTA and the
  // MMAs of every tile read them in place — no per-tile weight stream
  // competing with the operand reads for the shared-memory port, no
  // per-stage barrier round trips.
  const int groups = (taps + G - 1) / G;
  const bool resident = g.n_tiles == 1 && cblocks == 1 && groups <= STAGES;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 2);  // both MMA warps release a stage
    }
    for (int h = 0; h < kSlots; ++h) {
      // TMA: the producer's expect_tx arrival; GATHER: each gathering warp.
      tc::mbar_init(&hfull[h], GATHER ? kGatherThreads / 32 : 1);
      tc::mbar_init(&hempty[h], 2);
    }
    for (int a = 0; a < 4; ++a) {
      tc::mbar_init(&tfull[a], 1);
      // The block's epilogue warps (PAIR: of both CTAs, on rank 0's barrier).
      tc::mbar_init(&tempty[a], PAIR ? kEpilogueWarps : kEpilogueWarps / 2);
    }
    tc::mbar_init(&done[0], 1);
    tc::mbar_init(&done[1], 1);
    tmem_slot[1] = 0;  // epilogue abort flag (POOL)
    tc::fence_barrier_init();
    tc::prefetch_tmap(&tmW);
    if (!GATHER) tc::prefetch_tmap(&tmX);
  }
  if (warp == 1) {
    if (PAIR) {
      tc::tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
      tc::tmem_relinquish_pair();
    } else {
      tc::tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
      tc::tmem_relinquish();
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (PAIR) tc::cluster_sync();  // both CTAs' barriers initialised, TMEM allocated
  tc::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // the previous kernel's outputs are complete from here on

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer: input windows and weight tiles ----------------
      // PAIR: both CTAs load into their own shared memory at the same
      // offsets and count the bytes on rank 0's barriers, which rank 0
      // arms for both; weight rows [rank BN / 2, + BN / 2) of the tile.
      const uint32_t halo_bytes = (uint32_t)(hw * hh) * Cfg::ROW;
      constexpr uint32_t kCtas = PAIR ? 2 : 1;
      const bool arm = !PAIR || rank == 0;
      const int wrow = PAIR ? (int)rank * (BN / 2) : 0;
      auto load_w = [&](void* dst, uint64_t* bar, int x, int y) {
        if (PAIR)
          tc::tma_load_2d_pair(dst, &tmW, tc::mapa(tc::smem_u32(bar), 0), x, y + wrow);
        else
          tc::tma_load_2d(dst, &tmW, bar, x, y);
      };
      int stage = 0, hs = 0;
      uint32_t phase = 0, hphase = 0;
      bool ok = true;
      if (resident) {
        for (int grp = 0; grp < groups; ++grp) {
          const int t0 = grp * G, gt = taps - t0 < G ? taps - t0 : G;
          if (arm) tc::mbar_arrive_expect_tx(&full[grp], kCtas * gt * Cfg::B_BYTES);
          for (int j = 0; j < gt; ++j)
            load_w(smem + grp * Cfg::STAGE_BYTES + j * Cfg::B_BYTES, &full[grp], (t0 + j) * g.C4, 0);
        }
      }
      for (int64_t k = 0; ok; ++k) {
        const int64_t tile = halo_unit<POOL, PAIR>(g, k, rank).tile;
        if (tile < 0) break;
        const int64_t mt = tile / g.n_tiles;
        const int nt = (int)(tile % g.n_tiles);
        const int n = (int)(mt / per_img), rem = (int)(mt % per_img);
        const int y0 = (rem / g.tiles_x) * 2 * kHaloTH, x0 = (rem % g.tiles_x) * kHaloTW;
        for (int cb = 0; cb < cblocks && ok; ++cb) {
          if (!GATHER) {  // else the gathering warps fill the windows
            if (!tc::mbar_wait(&hempty[hs], hphase ^ 1, g.err)) {
              ok = false;
              break;
            }
            if (arm) tc::mbar_arrive_expect_tx(&hfull[hs], kCtas * halo_bytes);
            if (PAIR)
              tc::tma_load_4d_pair(halo + hs * Cfg::SLOT_BYTES, &tmX,
                                   tc::mapa(tc::smem_u32(&hfull[hs]), 0), cb * CB, x0 * g.sw - g.pw,
                                   y0 * g.sh - g.ph, n);
            else
              tc::tma_load_4d(halo + hs * Cfg::SLOT_BYTES, &tmX, &hfull[hs], cb * CB,
                              x0 * g.sw - g.pw, y0 * g.sh - g.ph, n);
            if (++hs == kSlots) {
              hs = 0;
              hphase ^= 1;
            }
          }
          for (int t0 = 0; t0 < taps && !resident; t0 += G) {
            const int gt = taps - t0 < G ? taps - t0 : G;
            if (!tc::mbar_wait(&empty[stage], phase ^ 1, g.err)) {
              ok = false;
              break;
            }
            if (arm) tc::mbar_arrive_expect_tx(&full[stage], kCtas * gt * Cfg::B_BYTES);
            for (int j = 0; j < gt; ++j)
              load_w(smem + stage * Cfg::STAGE_BYTES + j * Cfg::B_BYTES, &full[stage],
                     (t0 + j) * g.C4 + cb * CB, nt * BN);
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1;
            }
          }
        }
      }
      // Let the last issued loads land before the CTA can exit (PAIR: rank
      // 0's barriers count both CTAs' loads; rank 1 leaves only after the
      // final commit, which follows every MMA that read them).
      if (ok && resident && arm) {
        for (int grp = 0; grp < groups; ++grp) tc::mbar_wait(&full[grp], 0, g.err);
      }
      if (ok && arm) {
        for (int q = 0; q < STAGES && !resident; ++q) {
          if (stage == 0) {
            stage = STAGES;
            phase ^= 1;
          }
          --stage;
          tc::mbar_wait(&full[stage], phase, g.err);
        }
        for (int q = 0; q < kSlots && !GATHER; ++q) {
          if (hs == 0) {
            hs = kSlots;
            hphase ^= 1;
          }
          --hs;
          tc::mbar_wait(&hfull[hs], hphase, g.err);
        }
      }
    }
  } else if (warp <= 2 && PAIR && rank != 0) {
    // PAIR, rank 1: rank 0 issues; wait for its final commits before leaving.
    tc::mbar_wait_warp(&done[warp - 1], 0, g.err);
  } else if (warp <= 2) {
    // ---------------- MMA issuers: warp 1 upper block, warp 2 lower block ----------------
    // PAIR: M = 256 MMAs over both CTAs' windows and weight halves, into
    // both CTAs' accumulators; commits reach both CTAs' barriers.
    const int blk = warp - 1;
    constexpr uint32_t idesc = tc::idesc_tf32(PAIR ? 2 * BM : BM, BN);
    auto commit = [](uint64_t* bar) {
      if (PAIR)
        tc::mma_commit_pair_both(bar);
      else
        tc::mma_commit(bar);
    };
    // Descriptor start addresses are in 16-byte units: adding (bytes >> 4)
    // moves a descriptor (all shared addresses here are below 256 KB).
    const uint64_t a_desc0 =
        tc::desc_kmajor_swz(tc::smem_u32(halo), (uint32_t)hw * Cfg::ROW, Cfg::ROW) +
        (uint32_t)(blk * kHaloTH * hw) * (Cfg::ROW >> 4);
    const uint64_t b_desc0 = tc::desc_kmajor_swz(tc::smem_u32(smem), 8 * Cfg::ROW, Cfg::ROW);
    int stage = 0, hs = 0;
    uint32_t phase = 0, hphase = 0;
    bool ok = true;
    if (resident) {
      for (int grp = 0; grp < groups && ok; ++grp) ok = tc::mbar_wait_warp(&full[grp], 0, g.err);
      tc::tc_fence_after();
    }
    for (int64_t local = 0; ok && halo_unit<POOL, PAIR>(g, local, rank).tile >= 0; ++local) {
      const int acc = local & 1;
      const uint32_t aphase = (local >> 1) & 1;
      if (!tc::mbar_wait_warp(&tempty[acc * 2 + blk], aphase ^ 1, g.err)) break;
      tc::tc_fence_after();
      const uint32_t d_tmem = tmem_base + (uint32_t)(acc * 2 + blk) * BN;
      uint32_t accumulate = 0;  // the tile's first MMA overwrites the accumulator
      for (int cb = 0; cb < cblocks && ok; ++cb) {
        if (!tc::mbar_wait_warp(&hfull[hs], hphase, g.err)) {
          ok = false;
          break;
        }
        tc::tc_fence_after();
        const uint64_t a_win = a_desc0 + (uint32_t)hs * (Cfg::SLOT_BYTES >> 4);
        int kh = 0, kw = 0;
        for (int t0 = 0; t0 < taps; t0 += G) {
          const int gt = taps - t0 < G ? taps - t0 : G;
          if (resident) {
            stage = t0 / G;
          } else {
            if (!tc::mbar_wait_warp(&full[stage], phase, g.err)) {
              ok = false;
              break;
            }
            tc::tc_fence_after();
          }
          const uint64_t b_stage = b_desc0 + (uint32_t)stage * (Cfg::STAGE_BYTES >> 4);
          if (tc::elect_one()) {
            int th = kh, tw = kw;
            uint32_t accum = accumulate;
#pragma unroll
            for (int j = 0; j < G; ++j) {
              if (j < gt) {
                const uint64_t a = a_win + (uint32_t)(th * hw + tw) * (Cfg::ROW >> 4);
                const uint64_t b = b_stage + (uint32_t)j * (Cfg::B_BYTES >> 4);
#pragma unroll
                for (int k = 0; k < CB / 8; ++k) {
                  if (PAIR)
                    tc::mma_tf32_pair(d_tmem, a + 2 * k, b + 2 * k, idesc, accum);
                  else
                    tc::mma_tf32(d_tmem, a + 2 * k, b + 2 * k, idesc, accum);
                  accum = 1;
                }
                if (++tw == g.KW) {
                  tw = 0;
                  ++th;
                }
              }
            }
            if (!resident) commit(&empty[stage]);
          }
          __syncwarp();
          accumulate = 1;
          for (int j = 0; j < gt; ++j) {
            if (++kw == g.KW) {
              kw = 0;
              ++kh;
            }
          }
          if (!resident && ++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        // The window is free once both blocks' taps that read it completed.
        if (tc::elect_one()) commit(&hempty[hs]);
        __syncwarp();
        if (++hs == kSlots) {
          hs = 0;
          hphase ^= 1;
        }
      }
      if (tc::elect_one()) commit(&tfull[acc * 2 + blk]);
      __syncwarp();
    }
    if (tc::elect_one()) commit(&done[blk]);
    __syncwarp();
    tc::mbar_wait_warp(&done[blk], 0, g.err);
  } else if (GATHER && warp >= 3 + kEpilogueWarps) {
    // ---------------- GATHER: space-to-depth windows from the source ----------------
    const int p = threadIdx.x - 32 * (3 + kEpilogueWarps);
    const int rows = hw * hh;
    // 16-byte loads: unit column stride, rows, planes and images in 4-float
    // multiples from a 16-byte aligned base, window origins on even s2d
    // columns (tile columns are 8 apart: an even pad).
    const bool vec = g.src_sw == 1 && g.src_sh % 4 == 0 && g.src_sc % 4 == 0 &&
                     g.src_sn % 4 == 0 && (((uintptr_t)g.src) & 15) == 0 && g.pw % 2 == 0;
    int hs = 0;
    uint32_t hphase = 0;
    for (int64_t k = 0;; ++k) {
      const int64_t tile = halo_unit<POOL, false>(g, k, 0).tile;
      if (tile < 0) break;
      const int64_t mt = tile / g.n_tiles;
      const int n = (int)(mt / per_img), rem = (int)(mt % per_img);
      const int i0 = (rem / g.tiles_x) * 2 * kHaloTH - g.ph, j0 = (rem % g.tiles_x) * kHaloTW - g.pw;
      if (!tc::mbar_wait_warp(&hempty[hs], hphase ^ 1, g.err)) break;
      uint8_t* slot = halo + hs * Cfg::SLOT_BYTES;
      const float* src = g.src + (int64_t)n * g.src_sn;
      if (vec) {
        // NCHW rows of 4-float multiples: a work item is two neighbouring
        // window pixels (wx even), whose 2 x 2 source blocks of one channel
        // row are one 16-byte load: 6 loads per item, two items in flight.
        const int pw2 = (hw + 1) >> 1, items = hh * pw2;
#pragma unroll 1
        for (int it0 = p; it0 < items; it0 += 2 * kGatherThreads) {
          float4 d[2][3][2];  // [item][c][dy]: (dx 0, 1) of pixel wx, then of wx + 1
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int it = it0 + u * kGatherThreads;
            const int wy = it / pw2, wx = 2 * (it - (it / pw2) * pw2);
            const int Y0 = 2 * (i0 + wy), X0 = 2 * (j0 + wx);
            const bool whole = X0 >= 0 && X0 + 3 < g.src_W;
#pragma unroll
            for (int dy = 0; dy < 2; ++dy) {
              const int Y = Y0 + dy;
              const bool row_in = it < items && (unsigned)Y < (unsigned)g.src_H;
#pragma unroll
              for (int c = 0; c < 3; ++c) {
                const float* px = src + c * g.src_sc + Y * g.src_sh + X0;
                if (row_in && whole) {
                  d[u][c][dy] = __ldg(reinterpret_cast<const float4*>(px));
                } else {
                  float e[4];
#pragma unroll
                  for (int k = 0; k < 4; ++k)
                    e[k] = row_in && (unsigned)(X0 + k) < (unsigned)g.src_W ? __ldg(px + k) : 0.0f;
                  d[u][c][dy] = make_float4(e[0], e[1], e[2], e[3]);
                }
              }
            }
          }
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int it = it0 + u * kGatherThreads;
            if (it >= items) continue;
            const int wy = it / pw2, wx = 2 * (it - (it / pw2) * pw2);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              if (wx + h >= hw) continue;
              const int r = wy * hw + wx + h;
              // channel 3 q + c, q = 2 dy + dx: component 2 h + dx of d[c][dy]
              float v[12];
#pragma unroll
              for (int c = 0; c < 3; ++c)
#pragma unroll
                for (int dy = 0; dy < 2; ++dy) {
                  const float4 t = d[u][c][dy];
                  v[3 * (2 * dy) + c] = h ? t.z : t.x;
                  v[3 * (2 * dy + 1) + c] = h ? t.w : t.y;
                }
              float4* row = reinterpret_cast<float4*>(slot + r * 64);
              const int sw = (r >> 1) & 3;
              row[0 ^ sw] = make_float4(v[0], v[1], v[2], v[3]);
              row[1 ^ sw] = make_float4(v[4], v[5], v[6], v[7]);
              row[2 ^ sw] = make_float4(v[8], v[9], v[10], v[11]);
              row[3 ^ sw] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
          }
        }
      } else {
      // Up to four rows per thread in flight (the 4 x 4 stem window is
      // 35 x 11 = 385 rows for 128 threads: one pass).
#pragma unroll 1
      for (int r0 = p; r0 < rows; r0 += 4 * kGatherThreads) {
        float v[4][12];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int r = r0 + u * kGatherThreads;
          const int wy = r / hw, wx = r - (r / hw) * hw;
          const int Y0 = 2 * (i0 + wy), X0 = 2 * (j0 + wx);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int Y = Y0 + (q >> 1), X = X0 + (q & 1);
            const bool in = r < rows && (unsigned)Y < (unsigned)g.src_H && (unsigned)X < (unsigned)g.src_W;
            const float* px = src + Y * g.src_sh + X * g.src_sw;
#pragma unroll
            for (int c = 0; c < 3; ++c) v[u][3 * q + c] = in ? __ldg(px + c * g.src_sc) : 0.0f;
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int r = r0 + u * kGatherThreads;
          if (r < rows) {
            float4* row = reinterpret_cast<float4*>(slot + r * 64);
            const int sw = (r >> 1) & 3;
            row[0 ^ sw] = make_float4(v[u][0], v[u][1], v[u][2], v[u][3]);
            row[1 ^ sw] = make_float4(v[u][4], v[u][5], v[u][6], v[u][7]);
            row[2 ^ sw] = make_float4(v[u][8], v[u][9], v[u][10], v[u][11]);
            row[3 ^ sw] = make_float4(0.f, 0.f, 0.f, 0.f);
          }
        }
      }
      }
      tc::fence_proxy_async_smem();  // generic stores -> the MMAs' async-proxy reads
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&hfull[hs]);
      if (++hs == kSlots) {
        hs = 0;
        hphase ^= 1;
      }
    }
  } else {
    // ---------------- epilogue: warps 3..6 upper, 7..10 lower block ----------------
    const int e = warp - 3, blk = e >> 2, quad = warp & 3;
    float* stage_tile = epi + e * 32 * (kStageCols + 1);
    const bool vec_ok = (g.Cout % 4 == 0) && ((((uintptr_t)g.out) & 15) == 0) &&
                        (!g.residual || ((((uintptr_t)g.residual) & 15) == 0));
    const bool bias_vec = g.bias && ((((uintptr_t)g.bias) & 15) == 0);
    const bool direct = vec_ok && perm_rows(g.Cout) && g.direct_epi;
    const int64_t OHW = (int64_t)g.OH * g.OW;
    float* row_carry = reinterpret_cast<float*>(smem + Cfg::CARRY_OFF);
    float* col_carry = row_carry + kPoolMaxOW * Cfg::ROW_CARRY_STRIDE;
    uint32_t parity = 0;  // POOL: exchange-buffer alternation
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    // PAIR: both CTAs' epilogue warps release an accumulator on rank 0.
    const uint32_t tempty_bar = PAIR ? tc::mapa(tc::smem_u32(&tempty[0]), 0) : 0;
    for (int64_t local = 0;; ++local) {
      const HaloUnit hu = halo_unit<POOL, PAIR>(g, local, rank);
      const int64_t t = hu.tile;
      if (t < 0) break;
      const int64_t mt = t / g.n_tiles;
      const int nt = (int)(t % g.n_tiles);
      const int n = (int)(mt / per_img), rem = (int)(mt % per_img);
      const int acc = local & 1;
      const uint32_t aphase = (local >> 1) & 1;
      const bool ready = tc::mbar_wait(&tfull[acc * 2 + blk], aphase, g.err);
      if (POOL) {
        // The pooled epilogue synchronises the 8 warps: agree on giving up
        // (every wait above is bounded, so every warp gets here).
        if (!ready) *abort_flag = 1;
        epi_bar_sync();
        if (*abort_flag) break;
      } else if (!ready) {
        break;
      }
      tc::tc_fence_after();
      if (!hu.valid) {
        // PAIR: the neighbour's stand-in tile (never stored).
      } else if (POOL) {
        pool_tile<BN>(g, tmem_base, acc, blk, quad, lane, epi, row_carry, col_carry, parity, n,
                      (rem / g.tiles_x) * 2 * kHaloTH, (rem % g.tiles_x) * kHaloTW);
      } else {
        store_tile<BN, true, BlockRows, STAGED>(g, tmem_base, (uint32_t)(acc * 2 + blk) * BN, nt, quad, 0,
                                                kStageCols, lane,
                       stage_tile, vec_ok, bias_vec,
                       BlockRows{(int64_t)n * OHW, (rem / g.tiles_x) * 2 * kHaloTH + blk * kHaloTH,
                                 (rem % g.tiles_x) * kHaloTW, g.OH, g.OW},
                       direct);
      }
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (PAIR)
          tc::mbar_arrive_cluster(tempty_bar + (acc * 2 + blk) * (uint32_t)sizeof(uint64_t));
        else
          tc::mbar_arrive(&tempty[acc * 2 + blk]);
      }
    }
  }

  tc::tc_fence_before();
  __syncthreads();
  if (PAIR) tc::cluster_sync();  // neither CTA frees the pair's TMEM while the other works
  if (warp == 1) {
    tc::tc_fence_after();
    if (PAIR)
      tc::tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
    else
      tc::tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// ------------------------------------------------------ layout kernels ----

// OIHW -> [plane][Cout][K_pad], zero padded, rows in perm_col order when
// C_out is a multiple of 32. Chunk mode: k = (kh*KW + kw)*C4 + ci (C4 =
// channels padded to 32); element mode: k = (ci*KH + kh)*KW + kw, the OIHW
// order itself. split: plane 0 = tf32(w), plane 1 = w - tf32(w); else plane
// 0 = w.
__global__ void __launch_bounds__(256) pack_weight_kernel(const float* __restrict__ w,
                                                          float* __restrict__ out, int Cout,
                                                          int Cin, int KH, int KW, int C4,
                                                          int Kpad, int split, int element) {
  const int64_t total = (int64_t)Cout * Kpad;
  const int Kw = Cin * KH * KW;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / Kpad), k = (int)(i % Kpad);
    const int co = perm_rows(Cout) ? (r & ~31) + perm_col(r & 31) : r;
    float v = 0.0f;
    if (element) {
      if (k < Kw) v = w[(int64_t)co * Kw + k];
    } else {
      const int tap = k / C4, ci = k % C4;
      if (tap < KH * KW && ci < Cin) v = w[(((int64_t)co * Cin + ci) * KH + tap / KW) * KW + tap % KW];
    }
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
// One 32 x 32 (channel x pixel) tile per block: blockIdx.x pixel tile, y
// channel tile, z image (strided past 65535); no index division.
__global__ void __launch_bounds__(256) nchw_to_nhwc_pad_kernel(const float* __restrict__ x,
                                                               float* __restrict__ hi,
                                                               float* __restrict__ lo, int N, int C,
                                                               int64_t HW, int C4) {
  __shared__ float tile[32][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int64_t p0 = (int64_t)blockIdx.x * 32;
  const int c0 = blockIdx.y * 32;
  for (int64_t n = blockIdx.z; n < N; n += gridDim.z) {
#pragma unroll
    for (int j = ty; j < 32; j += 8) {
      const int c = c0 + j;
      const int64_t pix = p0 + tx;
      tile[j][tx] = (c < C && pix < HW) ? __ldg(x + (n * C + c) * HW + pix) : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int j = ty; j < 32; j += 8) {
      const int64_t pix = p0 + j;
      const int c = c0 + tx;
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

// NCHW [N][C][HW] -> NHWC [N][HW][C4] for C4 <= 16 (model inputs such as
// RGB): one thread per pixel, reads coalesced along each channel plane,
// writes C4 / 4 consecutive 16-byte vectors; optional hi/lo.
__global__ void __launch_bounds__(256) nchw_to_nhwc_small_kernel(const float* __restrict__ x,
                                                                 float* __restrict__ hi,
                                                                 float* __restrict__ lo, int N,
                                                                 int C, int64_t HW, int C4) {
  const int64_t total = (int64_t)N * HW;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = i / HW, p = i - n * HW;
    const float* src = x + n * C * HW + p;
    for (int c0 = 0; c0 < C4; c0 += 4) {
      float v[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) v[q] = (c0 + q < C) ? src[(int64_t)(c0 + q) * HW] : 0.0f;
      float4* dh = reinterpret_cast<float4*>(hi + i * C4 + c0);
      if (lo) {
        float h[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) h[q] = tc::to_tf32(v[q]);
        *dh = make_float4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<float4*>(lo + i * C4 + c0) =
            make_float4(v[0] - h[0], v[1] - h[1], v[2] - h[2], v[3] - h[3]);
      } else {
        *dh = make_float4(v[0], v[1], v[2], v[3]);
      }
    }
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

// How a weight of shape [Cout, Cin, KH, KW] is packed, decided by the shape
// alone (so a weight prepacked once matches every later call): chunk mode
// with channels padded to a multiple of 4, or element mode for tiny K.
// Space-to-depth input for stride-2 convolutions with few channels: output
// pixel (i, j) of [N][ceil(H/2)][ceil(W/2)][C2] (C2 = 16 or 32) holds, in
// channel q C + c (q = 2 dy + dx), input channel c at (2i + dy, 2j + dx)
// (zero past the image), and zeros in channels 4C..C2-1. Input strides in
// elements (NCHW or NHWC).
template <int C2>
__global__ void __launch_bounds__(256) s2d_input_kernel(const float* __restrict__ x,
                                                        float* __restrict__ out, int N, int C, int H,
                                                        int W, int H2, int W2, int64_t xs_n,
                                                        int64_t xs_c, int64_t xs_h, int64_t xs_w) {
  const int64_t total = (int64_t)N * H2 * W2;
  for (int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; p < total;
       p += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = p / ((int64_t)H2 * W2);
    const int rem = (int)(p - n * H2 * W2);
    const int i = rem / W2, j = rem - (rem / W2) * W2;
    float4* dst = reinterpret_cast<float4*>(out + p * C2);
#pragma unroll
    for (int k4 = 0; k4 < C2 / 4; ++k4) {
      float v[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int cc = 4 * k4 + e, q = cc / C, c = cc - q * C;
        const int y = 2 * i + (q >> 1), xx = 2 * j + (q & 1);
        v[e] = (q < 4 && y < H && xx < W) ? x[n * xs_n + c * xs_c + y * xs_h + xx * xs_w] : 0.0f;
      }
      dst[k4] = make_float4(v[0], v[1], v[2], v[3]);
    }
  }
}

// The same rewrite for an NCHW input, one output row (n, i) per block: the
// block stages input rows 2 i and 2 i + 1 of every channel in shared memory
// with coalesced loads (16-byte ones when VEC: W and the strides a multiple of
// 4 floats, an aligned base), then writes the row's W2 x C2 floats as
// consecutive 16-byte stores. A thread's float4 index inside a pixel is fixed
// (the block size is a multiple of C2 / 4), so its channel sources are too.
template <int C2, bool VEC>
__global__ void __launch_bounds__(128) s2d_rows_kernel(const float* __restrict__ x,
                                                       float* __restrict__ out, int C, int H, int W,
                                                       int H2, int W2, int64_t xs_n, int64_t xs_c,
                                                       int64_t xs_h) {
  extern __shared__ float rows[];  // [2 C][W]: row 2 c + dy = channel c, input row 2 i + dy
  pdl_trigger();
  pdl_wait();
  const int64_t row = blockIdx.x;  // n H2 + i
  const int n = (int)(row / H2), i = (int)(row - (int64_t)n * H2);
  const float* src = x + n * xs_n;
  if (VEC) {
    const int W4 = W >> 2;
    for (int idx = threadIdx.x; idx < 2 * C * W4; idx += blockDim.x) {
      const int rr = idx / W4, x4 = idx - rr * W4;
      const int y = 2 * i + (rr & 1);
      const float4 v = y < H ? __ldg(reinterpret_cast<const float4*>(src + (rr >> 1) * xs_c +
                                                                       (int64_t)y * xs_h) + x4)
                             : make_float4(0.f, 0.f, 0.f, 0.f);
      reinterpret_cast<float4*>(rows + rr * W)[x4] = v;
    }
  } else {
    for (int idx = threadIdx.x; idx < 2 * C * W; idx += blockDim.x) {
      const int rr = idx / W, xx = idx - rr * W;
      const int y = 2 * i + (rr & 1);
      rows[idx] = y < H ? __ldg(src + (rr >> 1) * xs_c + (int64_t)y * xs_h + xx) : 0.0f;
    }
  }
  __syncthreads();
  constexpr int P4 = C2 / 4;  // float4s per pixel
  const int k4 = threadIdx.x % P4;
  int off[4], dx[4];
  bool used[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int cc = 4 * k4 + e, q = cc / C, c = cc - q * C;
    used[e] = q < 4;
    dx[e] = q & 1;
    off[e] = (2 * c + (q >> 1)) * W + dx[e];
  }
  float4* dst = reinterpret_cast<float4*>(out + row * W2 * C2);
  for (int idx = threadIdx.x; idx < W2 * P4; idx += blockDim.x) {
    const int j = idx / P4;
    float v[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) v[e] = (used[e] && 2 * j + dx[e] < W) ? rows[off[e] + 2 * j] : 0.0f;
    dst[idx] = make_float4(v[0], v[1], v[2], v[3]);
  }
}

// Space-to-depth weights: [C_out][KH2][KW2][C2] in the halo kernel's k order,
// W'[co, kh2, kw2, q C + c] = W[co, c, 2 (kh2 - pad_h) + dy + ph,
// 2 (kw2 - pad_w) + dx + pw] inside the original window, else zero; rows in
// perm_col order like every packed weight. The source is the OIHW weight, or
// a prepacked one (chunk or element k order).
__global__ void __launch_bounds__(256) s2d_weight_kernel(const float* __restrict__ w,
                                                         float* __restrict__ out, int Cout, int C,
                                                         int KH, int KW, int ph, int pw, int KH2,
                                                         int KW2, int pad_h, int pad_w, int src_mode,
                                                         int src_c4, int src_kpad, int C2) {
  pdl_trigger();
  pdl_wait();
  const int64_t total = (int64_t)Cout * KH2 * KW2 * C2;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int cc = (int)(i % C2);
    const int64_t t = i / C2;
    const int kw2 = (int)(t % KW2), kh2 = (int)((t / KW2) % KH2);
    const int co = (int)(t / ((int64_t)KW2 * KH2));
    const int q = cc / C, c = cc - q * C;
    const int kh = 2 * (kh2 - pad_h) + (q >> 1) + ph, kw = 2 * (kw2 - pad_w) + (q & 1) + pw;
    float v = 0.0f;
    if (q < 4 && kh >= 0 && kh < KH && kw >= 0 && kw < KW) {
      // Row co holds channel perm_col order (a prepacked source row already does).
      const int ch = perm_rows(Cout) ? (co & ~31) + perm_col(co & 31) : co;
      if (src_mode == 0)  // OIHW
        v = w[(((int64_t)ch * C + c) * KH + kh) * KW + kw];
      else if (src_mode == 1)  // prepacked, chunk order k = (kh KW + kw) C4 + c
        v = w[(int64_t)co * src_kpad + (kh * KW + kw) * src_c4 + c];
      else  // prepacked, element order k = (c KH + kh) KW + kw
        v = w[(int64_t)co * src_kpad + (c * KH + kh) * KW + kw];
    }
    out[i] = v;
  }
}

// ---------------------------------------------------- direct small conv ----
// Convolutions with few output channels and a short reduction (C_out <= 16,
// C KH KW <= 256: LeNet's 1 -> 6 and 6 -> 16 5x5 layers) on the CUDA cores:
// a tensor-core tile would be mostly padding (N >= 64 of 16 channels, K
// padded to 32), and the work is an HBM-bound stencil. One thread per output
// pixel holds all C_out accumulators; each block stages the weights once in
// shared memory as [c][kh][kw][co] (CO floats per tap, read by every thread
// at the same address: a broadcast) in full fp32 (hi + lo planes of a
// prepacked weight). Accumulation is fp32 FMA over k = (c, kh, kw), the
// reference's order; bias, residual and activation as in store_tile.
constexpr int kDirectMaxK = 256;
// Stages the C_out x K weight in shared memory as ws[k * CO + co] (zero for
// co >= C_out) from OIHW (src_mode 0) or a prepacked [hi, lo][C_out][K_pad]
// weight in chunk (1) or element (2) order.
template <int CO>
__device__ __forceinline__ void stage_direct_weights(const ConvArgs& g, const float* __restrict__ w,
                                                     int src_mode, int src_c4, int src_kpad,
                                                     float* ws) {
  const int K = g.K;  // C KH KW
  for (int idx = threadIdx.x; idx < K * CO; idx += blockDim.x) {
    const int k = idx / CO, co = idx - k * CO;
    float v = 0.0f;
    if (co < g.Cout) {
      const int c = k / (g.KH * g.KW), t = k - c * (g.KH * g.KW);
      if (src_mode == 0) {
        v = w[(int64_t)co * K + k];
      } else {
        const int64_t off = (int64_t)co * src_kpad + (src_mode == 1 ? t * src_c4 + c : k);
        v = __fadd_rn(w[off], w[(int64_t)g.Cout * src_kpad + off]);
      }
    }
    ws[k * CO + co] = v;
  }
}

// Writes one output pixel's channels: bias, residual (conv+add+relu), activation.
template <int CO>
__device__ __forceinline__ void direct_store(const ConvArgs& g, const float (&acc)[CO], int64_t m,
                                             int64_t n, int64_t p, int64_t OHW, int co0 = 0) {
  const bool add = g.act == kActAddRelu;
#pragma unroll
  for (int j = 0; j < CO; ++j) {
    const int co = co0 + j;
    if (co >= g.Cout) break;
    const int64_t off = g.out_nhwc ? m * g.Cout + co : (n * g.Cout + co) * OHW + p;
    float o = acc[j];
    if (g.bias) o = __fadd_rn(o, __ldg(g.bias + co));
    if (add) o = __fadd_rn(o, __ldg(g.residual + off));
    g.out[off] = activate(o, g.act);
  }
}

template <int CO>
__global__ void __launch_bounds__(128) conv_direct_kernel(ConvArgs g, const float* __restrict__ w,
                                                          int src_mode, int src_c4, int src_kpad) {
  __shared__ __align__(16) float ws[kDirectMaxK * CO];
  const int C = g.K / (g.KH * g.KW);
  stage_direct_weights<CO>(g, w, src_mode, src_c4, src_kpad, ws);
  __syncthreads();
  const int64_t OHW = (int64_t)g.OH * g.OW;
  for (int64_t m = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; m < g.M;
       m += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = m / OHW;
    const int p = (int)(m - n * OHW);
    const int oh = p / g.OW, ow = p - oh * g.OW;
    const int ih0 = oh * g.sh - g.ph, iw0 = ow * g.sw - g.pw;
    float acc[CO];
#pragma unroll
    for (int co = 0; co < CO; ++co) acc[co] = 0.0f;
    // Element offsets stay 32-bit inside one image (host-checked).
    const float* xn = g.x_hi + n * g.xs_n;
    const int sc = (int)g.xs_c, shh = (int)g.xs_h, sww = (int)g.xs_w;
    const float4* wk = reinterpret_cast<const float4*>(ws);
    for (int c = 0; c < C; ++c) {
      const float* xc = xn + c * sc;
      for (int kh = 0; kh < g.KH; ++kh) {
        const int ih = ih0 + kh;
        const bool row_ok = (unsigned)ih < (unsigned)g.H;
        const float* xr = xc + ih * shh;
        for (int kw = 0; kw < g.KW; ++kw, wk += CO / 4) {
          const int iw = iw0 + kw;
          const float xv = (row_ok && (unsigned)iw < (unsigned)g.W) ? __ldg(xr + iw * sww) : 0.0f;
#pragma unroll
          for (int q = 0; q < CO / 4; ++q) {
            const float4 wv = wk[q];
            acc[4 * q] = fmaf(xv, wv.x, acc[4 * q]);
            acc[4 * q + 1] = fmaf(xv, wv.y, acc[4 * q + 1]);
            acc[4 * q + 2] = fmaf(xv, wv.z, acc[4 * q + 2]);
            acc[4 * q + 3] = fmaf(xv, wv.w, acc[4 * q + 3]);
          }
        }
      }
    }
    direct_store<CO>(g, acc, m, n, p, OHW);
  }
}

// ------------------------------------------- small conv on tensor cores ----
// The same calls (C_out <= 16) in TF32 mode with many output pixels and a
// reduction of at most 160 over at most 32 window taps (LeNet's layers at
// batch 8192): one M = 128 pixels x N = 16 channels tcgen05 tile per step.
// The CTA's threads build the tile's im2col rows in shared memory themselves
// (a few channels per pixel are too narrow for TMA im2col): row r is output
// pixel m0 + r, K-major in 32-float k-blocks under the 128-byte swizzle
// (16-byte chunk j of row r at j ^ (r & 7)); TPR threads share a row, one
// k-block each in turn. The k order is the reference's (c, kh, kw), or (kh,
// kw, c) for channels-last inputs with an even channel count, whose channel
// pairs then load as float2; the weight (zero rows up to 16 channels, zero k
// up to the k-blocks) is staged once per CTA in the same order. Each element
// reads its input offset and window-tap bit from per-k tables passed by value
// (constant-bank operands of the unrolled loads); a pixel's bit mask of
// in-bounds taps turns padding and k past K into zeros. Two row buffers and
// two 16-column TMEM accumulators pipeline the tiles: the MMAs of tile i run
// while the threads drain tile i - 1 (bias, residual, activation) and build
// tile i + 1.
constexpr int64_t kSmallTcMinM = 148 * 128 * 2;  // at least two tiles per SM
constexpr int kSmallTcMaxK = 160;                // five k-blocks

// Unsigned division by a launch constant d as a multiply and shift
// (Granlund and Montgomery, "Division by invariant integers using
// multiplication", PLDI 1994, round-up method with N = 32): l = ceil(log2 d),
// mul = floor(2^32 (2^l - d) / d) + 1, n / d = (umulhi(n, mul) + n) >> l for
// every 32-bit n.
struct FastDiv {
  unsigned mul, shift;
};
inline FastDiv fast_div(unsigned d) {
  unsigned l = 0;
  while ((1ull << l) < d) ++l;
  return {(unsigned)((((1ull << 32) * ((1ull << l) - d)) / d) + 1), l};
}
__device__ __forceinline__ unsigned fast_div(unsigned n, FastDiv f) {
  return (unsigned)(((uint64_t)__umulhi(n, f.mul) + n) >> f.shift);
}

struct SmallTcTable {
  int off[kSmallTcMaxK];       // input element offset of k from the window origin
  unsigned bit[kSmallTcMaxK];  // 1 << (kh KW + kw) of k; 0 past K
  FastDiv ohw, ow;             // pixel -> (image, row, column)
  int stage;                   // channels-last output through shared memory (16-byte aligned)
};

template <int KB>
struct SmallTcCfg {
  static constexpr int TPR = KB;                        // threads per row: one k-block each
  static constexpr int THREADS = 128 * TPR;
  static constexpr int EPI = TPR < 4 ? TPR : 4;         // warp groups sharing the epilogue
  static constexpr int MIN_CTAS = KB == 1 ? 6 : KB == 2 ? 3 : 1;  // resident by shared memory
  static constexpr uint32_t A_BYTES = KB * 128 * 128;  // one tile: KB k-blocks of 128 rows x 128 B
  static constexpr uint32_t B_BYTES = KB * 16 * 128;   // KB k-blocks of 16 rows x 128 B
  static constexpr uint32_t BAR_OFF = 2 * A_BYTES + B_BYTES;
  static constexpr size_t SMEM = (size_t)BAR_OFF + 64 + 1024;
};

template <int KB, bool VEC2>
__global__ void __launch_bounds__(SmallTcCfg<KB>::THREADS, SmallTcCfg<KB>::MIN_CTAS) conv_small_tc_kernel(
    const __grid_constant__ ConvArgs g, const __grid_constant__ SmallTcTable tab,
    const float* __restrict__ w, int src_mode, int src_c4, int src_kpad) {
  using Cfg = SmallTcCfg<KB>;
  constexpr int KP = KB * 32;
  constexpr int TPR = Cfg::TPR, EPI = Cfg::EPI, EPC = 16 / EPI;  // epilogue channels per group
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sb = smem + 2 * Cfg::A_BYTES;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + Cfg::BAR_OFF);  // [2]: MMAs of a buffer done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 2);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = threadIdx.x & 127, part = threadIdx.x >> 7;
  const int K = g.K, KHW = g.KH * g.KW, C = K / KHW;

  for (int idx = threadIdx.x; idx < 16 * KP; idx += Cfg::THREADS) {
    const int co = idx / KP, k = idx - co * KP;
    float v = 0.0f;
    if (co < g.Cout && k < K) {
      const int c = VEC2 ? k % C : k / KHW, t = VEC2 ? k / C : k % KHW;
      if (src_mode == 0) {
        v = w[(int64_t)co * K + c * KHW + t];
      } else {
        const int64_t off = (int64_t)co * src_kpad + (src_mode == 1 ? t * src_c4 + c : c * KHW + t);
        v = __fadd_rn(w[off], w[(int64_t)g.Cout * src_kpad + off]);
      }
    }
    const int kb = k >> 5, j = (k >> 2) & 7;
    *reinterpret_cast<float*>(sb + kb * 2048 + co * 128 + ((j ^ (co & 7)) << 4) + (k & 3) * 4) = v;
  }
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar[0], 1);
    tc::mbar_init(&bar[1], 1);
    tc::fence_barrier_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(tmem_slot, 32);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  constexpr uint32_t idesc = tc::idesc_tf32(BM, 16);
  const int OHW = g.OH * g.OW, M = (int)g.M, Cout = g.Cout;
  const int tiles = (M + BM - 1) / BM;
  unsigned rep = 0;  // bit kh KW for every kh: one bit per window row
  for (int kh = 0; kh < g.KH; ++kh) rep |= 1u << (kh * g.KW);
  float bias[EPC];  // this thread's epilogue channels
#pragma unroll
  for (int j = 0; j < EPC; ++j) {
    const int co = (part < EPI ? part : 0) * EPC + j;
    bias[j] = g.bias && co < Cout ? __ldg(g.bias + co) : 0.0f;
  }
  const bool add = g.act == kActAddRelu;
  bool ok = true;
  int prev = -1, i = 0;  // tile whose MMAs are in flight; this CTA's step
  for (int tile = blockIdx.x;; tile += gridDim.x, ++i) {
    const bool have = tile < tiles;
    const int buf = (int)(i & 1);
    if (have) {
      // This thread's k-blocks of row r (zeros past the last pixel).
      const int m = (int)tile * BM + r;  // pixel indices stay 32-bit (host-checked)
      unsigned taps = 0;
      const float* xn = g.x_hi;
      if (m < M) {
        const int n = (int)fast_div((unsigned)m, tab.ohw), p = m - n * OHW;
        const int oh = (int)fast_div((unsigned)p, tab.ow), ow = p - oh * g.OW;
        const int ih0 = oh * g.sh - g.ph, iw0 = ow * g.sw - g.pw;
        // In-bounds taps: kw in [c_lo, c_hi) of every kh in [r_lo, r_hi); the
        // product places the column mask at each such row's bit offset.
        const int c_lo = max(0, -iw0), c_hi = min(g.KW, g.W - iw0);
        const int r_lo = max(0, -ih0), r_hi = min(g.KH, g.H - ih0);
        if (c_hi > c_lo && r_hi > r_lo) {
          const unsigned cols = (unsigned)((1ull << c_hi) - (1ull << c_lo));
          const unsigned rows = rep & (unsigned)((1ull << (r_hi * g.KW)) - (1ull << (r_lo * g.KW)));
          taps = cols * rows;
        }
        xn = g.x_hi + (int64_t)n * g.xs_n + (int64_t)ih0 * g.xs_h + (int64_t)iw0 * g.xs_w;
      }
      uint8_t* row = smem + buf * Cfg::A_BYTES + r * 128;
#pragma unroll
      for (int kb = 0; kb < KB; ++kb) {
        if (kb % TPR != part) continue;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int k = kb * 32 + j * 4;
          float4 v;
          if constexpr (VEC2) {
            float2 lo = make_float2(0.0f, 0.0f), hi = make_float2(0.0f, 0.0f);
            if (taps & tab.bit[k]) lo = __ldg(reinterpret_cast<const float2*>(xn + tab.off[k]));
            if (taps & tab.bit[k + 2]) hi = __ldg(reinterpret_cast<const float2*>(xn + tab.off[k + 2]));
            v = make_float4(lo.x, lo.y, hi.x, hi.y);
          } else {
            v.x = (taps & tab.bit[k]) ? __ldg(xn + tab.off[k]) : 0.0f;
            v.y = (taps & tab.bit[k + 1]) ? __ldg(xn + tab.off[k + 1]) : 0.0f;
            v.z = (taps & tab.bit[k + 2]) ? __ldg(xn + tab.off[k + 2]) : 0.0f;
            v.w = (taps & tab.bit[k + 3]) ? __ldg(xn + tab.off[k + 3]) : 0.0f;
          }
          *reinterpret_cast<float4*>(row + kb * 16384 + ((j ^ (r & 7)) << 4)) = v;
        }
      }
      tc::fence_proxy_async_smem();  // the rows -> the MMAs' async-proxy reads
    }
    tc::tc_fence_before();
    // Every thread leaves the loop together if a wait gave up.
    ok = __syncthreads_and(ok ? 1 : 0) != 0;
    if (!ok) break;
    if (have && warp == 0) {
      tc::tc_fence_after();
      if (tc::elect_one()) {
        const uint32_t a0 = tc::smem_u32(smem + buf * Cfg::A_BYTES), b0 = tc::smem_u32(sb);
#pragma unroll
        for (int kb = 0; kb < KB; ++kb)
#pragma unroll
          for (int k = 0; k < 4; ++k)
            tc::mma_tf32(tmem_base + buf * 16, tc::desc_kmajor_sw128(a0 + kb * 16384 + k * 32),
                         tc::desc_kmajor_sw128(b0 + kb * 2048 + k * 32), idesc, (kb | k) != 0);
        tc::mma_commit(&bar[buf]);
      }
      __syncwarp();
    }
    if (prev >= 0) {
      // Drain the previous tile (buffer buf ^ 1, its (i - 1) / 2-th use).
      // Its row buffer, read by those MMAs, stages a channels-last output:
      // the tile's pixels are one contiguous range there, written back with
      // coalesced float4 stores (residual and activation on the way).
      ok = tc::mbar_wait_warp(&bar[buf ^ 1], (uint32_t)(((i - 1) >> 1) & 1), g.err);
      tc::tc_fence_after();
      const int m0 = prev * BM;
      float* obuf = reinterpret_cast<float*>(smem + (buf ^ 1) * Cfg::A_BYTES);
      if (ok && part < EPI) {
        uint32_t acc_bits[16];
        tc::tmem_ld16(tmem_base + (uint32_t)((buf ^ 1) * 16) + ((uint32_t)((warp & 3) * 32) << 16),
                      acc_bits);
        tc::tmem_ld_wait();
        const int rr = (warp & 3) * 32 + lane, m = m0 + rr;
        if (m < M) {
          // Channels [part EPC, part EPC + EPC): bias, then (unstaged)
          // residual and activation.
          const int n = (int)fast_div((unsigned)m, tab.ohw), p = m - n * OHW;
#pragma unroll
          for (int j = 0; j < EPC; ++j) {
            const int co = part * EPC + j;
            if (co >= Cout) break;
            uint32_t v = acc_bits[j];
#pragma unroll
            for (int q = 1; q < EPI; ++q) v = part == q ? acc_bits[q * EPC + j] : v;
            float o = __uint_as_float(v);
            if (g.bias) o = __fadd_rn(o, bias[j]);
            if (tab.stage) {
              obuf[rr * Cout + co] = o;
            } else {
              const int64_t off = g.out_nhwc ? (int64_t)m * Cout + co : ((int64_t)n * Cout + co) * OHW + p;
              if (add) o = __fadd_rn(o, __ldg(g.residual + off));
              g.out[off] = activate(o, g.act);
            }
          }
        }
      }
      if (tab.stage) {
        __syncthreads();
        const int nf = min(BM, M - m0) * Cout;
        float* out = g.out + (int64_t)m0 * Cout;
        const float* res = add ? g.residual + (int64_t)m0 * Cout : nullptr;
        for (int q = threadIdx.x * 4; q < nf; q += Cfg::THREADS * 4) {
          if (q + 4 <= nf) {
            float4 v = *reinterpret_cast<const float4*>(obuf + q);
            if (add) {
              const float4 rv = __ldg(reinterpret_cast<const float4*>(res + q));
              v.x = __fadd_rn(v.x, rv.x);
              v.y = __fadd_rn(v.y, rv.y);
              v.z = __fadd_rn(v.z, rv.z);
              v.w = __fadd_rn(v.w, rv.w);
            }
            v.x = activate(v.x, g.act);
            v.y = activate(v.y, g.act);
            v.z = activate(v.z, g.act);
            v.w = activate(v.w, g.act);
            *reinterpret_cast<float4*>(out + q) = v;
          } else {
            for (int e = q; e < nf; ++e) {
              float o = obuf[e];
              if (add) o = __fadd_rn(o, __ldg(res + e));
              out[e] = activate(o, g.act);
            }
          }
        }
        __syncthreads();  // the next step rebuilds this buffer's rows
      }
    }
    prev = have ? tile : -1;
    if (!have) break;
  }
  // After a wait gave up, the last issued MMAs (step i - 1) may still be in
  // flight: wait for them (bounded) before the accumulators are freed.
  if (!ok && prev >= 0) tc::mbar_wait(&bar[(i - 1) & 1], (uint32_t)(((i - 1) >> 1) & 1), nullptr);
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem_base, 32);
  }
}

// Stride-1-wide variant for a compile-time window width KW: a thread computes
// OWB horizontally adjacent output pixels of one row for CO of the CO * CG
// staged channels (CG threads, adjacent in the grid, share a pixel block),
// loading each input row segment (OWB - 1 + KW values) once per (channel,
// kh) into registers and reusing it across the KW taps. CG > 1 keeps the
// accumulators (OWB x CO) small enough for several blocks per SM. Same
// summation order per output as conv_direct_kernel (channel, kh, kw).
template <int CO, int CG, int KW, int OWB>
__global__ void __launch_bounds__(128, 5) conv_direct_row_kernel(ConvArgs g,
                                                                 const float* __restrict__ w,
                                                                 int src_mode, int src_c4,
                                                                 int src_kpad) {
  constexpr int CS = CO * CG;  // staged channels
  constexpr int kPix = 128 / CG * OWB;  // output pixels of one block pass
  __shared__ __align__(16) float ws[kDirectMaxK * CS];
  // Channels-last outputs leave through this buffer: the pass's pixels form
  // one contiguous range, written with coalesced stores (a thread's own
  // pixels are CO * OWB scattered scalars otherwise).
  __shared__ __align__(16) float obuf[kPix * CS];
  constexpr int XW = OWB - 1 + KW;
  constexpr int XW4 = (XW + 3) / 4;
  const int C = g.K / (g.KH * KW);
  stage_direct_weights<CS>(g, w, src_mode, src_c4, src_kpad, ws);
  __syncthreads();
  const int64_t OHW = (int64_t)g.OH * g.OW;
  const int nb = (g.OW + OWB - 1) / OWB;
  // 16-byte row reads need an aligned base, row and plane pitches that are
  // multiples of 4 floats, and a left pad that keeps ow0 - pw aligned.
  const bool x_vec = ((uintptr_t)g.x_hi & 15) == 0 && g.xs_h % 4 == 0 && g.xs_c % 4 == 0 &&
                     g.xs_n % 4 == 0 && g.pw % 4 == 0;
  // Unit and row indices are 32-bit (the host checks N * OH * nb * CG < 2^31):
  // 64-bit divisions cost ~70 instructions each here.
  const unsigned units = (unsigned)g.N * g.OH * nb * CG;
  const int sc = (int)g.xs_c, shh = (int)g.xs_h, sww = (int)g.xs_w;
  const bool staged = g.out_nhwc && g.Cout <= CS;
  const bool add = g.act == kActAddRelu;
  // Block-uniform passes (every thread takes part in the barriers).
  for (unsigned base = blockIdx.x * blockDim.x; base < units; base += gridDim.x * blockDim.x) {
    const unsigned u = base + threadIdx.x;
    const bool active = u < units;
    const int cg = (int)(u % CG);
    const unsigned ub = u / CG;
    const unsigned row = ub / nb;  // n * OH + oh
    const int ob = (int)(ub - row * nb);
    const unsigned n = row / g.OH;
    const int oh = (int)(row - n * g.OH);
    const int ow0 = ob * OWB;
    float acc[OWB][CO];
#pragma unroll
    for (int o = 0; o < OWB; ++o)
#pragma unroll
      for (int co = 0; co < CO; ++co) acc[o][co] = 0.0f;
    if (active) {
      const int ih0 = oh * g.sh - g.ph, iw0 = ow0 - g.pw;
      const float* xn = g.x_hi + (int64_t)n * g.xs_n;
      // Unit-stride rows whose segment starts 16-byte aligned and lies inside
      // the image width (planar input, W and the pad multiples of 4).
      const bool vec_rows = sww == 1 && iw0 >= 0 && iw0 + XW4 * 4 <= g.W && x_vec;
      const float4* wk = reinterpret_cast<const float4*>(ws) + cg * (CO / 4);
      for (int c = 0; c < C; ++c) {
        const float* xc = xn + c * sc;
        for (int kh = 0; kh < g.KH; ++kh, wk += KW * (CS / 4)) {
          const int ih = ih0 + kh;
          const bool row_ok = (unsigned)ih < (unsigned)g.H;
          const float* xr = xc + ih * shh;
          float xv[XW4 * 4];
          if (vec_rows) {  // the whole segment inside the row: 16-byte loads
#pragma unroll
            for (int j = 0; j < XW4; ++j) {
              float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
              if (row_ok) t = __ldg(reinterpret_cast<const float4*>(xr + iw0) + j);
              xv[4 * j] = t.x;
              xv[4 * j + 1] = t.y;
              xv[4 * j + 2] = t.z;
              xv[4 * j + 3] = t.w;
            }
          } else {
#pragma unroll
            for (int j = 0; j < XW; ++j) {
              const int iw = iw0 + j;
              xv[j] = (row_ok && (unsigned)iw < (unsigned)g.W) ? __ldg(xr + iw * sww) : 0.0f;
            }
          }
#pragma unroll
          for (int kw = 0; kw < KW; ++kw)
#pragma unroll
            for (int q = 0; q < CO / 4; ++q) {
              const float4 wv = wk[kw * (CS / 4) + q];
#pragma unroll
              for (int o = 0; o < OWB; ++o) {
                const float xo = xv[o + kw];
                acc[o][4 * q] = fmaf(xo, wv.x, acc[o][4 * q]);
                acc[o][4 * q + 1] = fmaf(xo, wv.y, acc[o][4 * q + 1]);
                acc[o][4 * q + 2] = fmaf(xo, wv.z, acc[o][4 * q + 2]);
                acc[o][4 * q + 3] = fmaf(xo, wv.w, acc[o][4 * q + 3]);
              }
            }
        }
      }
    }
    if (!staged) {
      if (active) {
#pragma unroll
        for (int o = 0; o < OWB; ++o) {
          const int ow = ow0 + o;
          if (ow >= g.OW) break;
          direct_store<CO>(g, acc[o], (int64_t)row * g.OW + ow, n, (int64_t)oh * g.OW + ow, OHW,
                           cg * CO);
        }
      }
      continue;  // block-uniform
    }
    // The pass's pixel range [m0, m1): from its first unit to its last.
    const unsigned ub0 = base / CG;
    const unsigned row0 = ub0 / nb;
    const int64_t m0 = (int64_t)row0 * g.OW + (int64_t)(ub0 - row0 * nb) * OWB;
    const unsigned u_last = (base + blockDim.x < units ? base + blockDim.x : units) - 1;
    const unsigned ubl = u_last / CG;
    const unsigned rowl = ubl / nb;
    const int owl = (int)(ubl - rowl * nb) * OWB + OWB;
    const int64_t m1 = (int64_t)rowl * g.OW + (owl < g.OW ? owl : g.OW);
    if (active) {
#pragma unroll
      for (int o = 0; o < OWB; ++o) {
        const int ow = ow0 + o;
        if (ow >= g.OW) break;
        const int pl = (int)((int64_t)row * g.OW + ow - m0);
#pragma unroll
        for (int j = 0; j < CO; ++j) {
          const int co = cg * CO + j;
          if (co < g.Cout)
            obuf[pl * g.Cout + co] = g.bias ? __fadd_rn(acc[o][j], __ldg(g.bias + co)) : acc[o][j];
        }
      }
    }
    __syncthreads();
    const int total = (int)(m1 - m0) * g.Cout;
    float* dst = g.out + m0 * g.Cout;
    const float* res = add ? g.residual + m0 * g.Cout : nullptr;
    int i0 = 0;
    if ((((uintptr_t)dst | (uintptr_t)res) & 15) == 0) {  // 16-byte runs, scalar tail
      const int n4 = total >> 2;
      for (int i = threadIdx.x; i < n4; i += blockDim.x) {
        float4 o = reinterpret_cast<const float4*>(obuf)[i];
        if (add) {
          const float4 r = __ldg(reinterpret_cast<const float4*>(res) + i);
          o.x = __fadd_rn(o.x, r.x);
          o.y = __fadd_rn(o.y, r.y);
          o.z = __fadd_rn(o.z, r.z);
          o.w = __fadd_rn(o.w, r.w);
        }
        o.x = activate(o.x, g.act);
        o.y = activate(o.y, g.act);
        o.z = activate(o.z, g.act);
        o.w = activate(o.w, g.act);
        reinterpret_cast<float4*>(dst)[i] = o;
      }
      i0 = n4 << 2;
    }
    for (int i = i0 + threadIdx.x; i < total; i += blockDim.x) {
      float o = obuf[i];
      if (add) o = __fadd_rn(o, __ldg(res + i));
      dst[i] = activate(o, g.act);
    }
    __syncthreads();  // obuf is rewritten by the next pass
  }
}

struct WeightLayout {
  int element;
  int C4;    // chunk mode: channels per tap as stored (multiple of 4)
  int K;     // valid k extent
  int Kpad;  // multiple of 32
};

WeightLayout weight_layout(int Cin, int KH, int KW) {
  WeightLayout L;
  const int ke = (int)cdiv((int64_t)Cin * KH * KW, BK) * BK;
  // Element order only for a single-k-block-or-two reduction (e.g. LeNet's
  // 1x5x5 conv), where padding channels to 4 would multiply the K work. A
  // 1 x 1 window over a multiple of 4 channels has the same k order and size
  // in both layouts, so it takes the chunk order (and the TMA paths).
  L.element = ke <= 64 && !(KH == 1 && KW == 1 && Cin % 4 == 0);
  if (L.element) {
    L.C4 = Cin;
    L.K = Cin * KH * KW;
    L.Kpad = ke;
  } else {
    L.C4 = (Cin + 3) / 4 * 4;
    L.K = KH * KW * L.C4;
    L.Kpad = (int)cdiv(L.K, BK) * BK;
  }
  return L;
}

// Which channels-last epilogues store straight from TMEM fragments:
// NNC_CUDA_CONV_DIRECT_EPI unset or 1 = the default policy (halo_direct),
// 0 = none (shared-memory staged stores, for comparison), 2 = every eligible
// call including 1 x 1 windows (for comparison).
static int direct_epilogue_mode() {
  static const int mode = [] {
    const char* e = getenv("NNC_CUDA_CONV_DIRECT_EPI");
    return e && e[0] == '0' ? 0 : (e && e[0] == '2' ? 2 : 1);
  }();
  return mode;
}
static bool direct_epilogue() { return direct_epilogue_mode() != 0; }

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
  // Activation im2col maps over the NHWC input: bounding box = window
  // origins of all output pixels, [-pad, (O-1)*stride - pad] per axis.
  CUtensorMap tx0 = tw0, tx1 = tw0;
  if (g.mode == kIm2col128 || g.mode == kIm2col16) {
    const uint64_t xd[4] = {(uint64_t)g.C4, (uint64_t)g.W, (uint64_t)g.H, (uint64_t)g.N};
    const uint64_t xs[3] = {(uint64_t)g.C4 * 4, (uint64_t)g.W * g.C4 * 4,
                            (uint64_t)g.H * g.W * g.C4 * 4};
    const int lower = -g.ph, upper = (g.OH - 1) * g.sh - g.ph - (g.H - 1);
    const bool sw128 = g.mode == kIm2col128;
    const uint32_t cpp = sw128 ? 32 : 4;
    if (!encode_tmap_im2col_f32(&tx0, g.x_hi, xd, xs, lower, upper, cpp, BM, g.sh, sw128, op))
      return false;
    tx1 = tx0;
    if (SPLIT == 2 &&
        !encode_tmap_im2col_f32(&tx1, g.x_lo, xd, xs, lower, upper, cpp, BM, g.sh, sw128, op))
      return false;
  }
  g.n_tiles = (int)cdiv(g.Cout, BN);
  g.m_tiles = (int)cdiv(g.M, BM);
  g.tiles = (int64_t)g.m_tiles * g.n_tiles;
  auto kern = conv_tc_kernel<BN, SPLIT, STAGES>;
  // The dynamic shared-memory opt-in is a property of the function in each
  // device's context: set it once per instantiation and device.
  static bool attr_set[64] = {};
  if (!attr_set[ctx().device]) {
    if (!check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)Cfg::SMEM),
                    op, "cudaFuncSetAttribute"))
      return false;
    attr_set[ctx().device] = true;
  }
  const int grid = (int)(g.tiles < sm_count() ? g.tiles : sm_count());
  g.direct_epi = direct_epilogue() ? 1 : 0;
  launch_pdl(kern, grid, kConvThreads, Cfg::SMEM, tw0, tw1, tx0, tx1, g);
  return check_launch(op);
}

// Whether the im2col route runs C_out > 64 on CTA pairs (the default);
// NNC_CUDA_CONV_PAIR=0 selects the single-CTA kernel (for comparison).
static bool conv_pair_enabled() {
  static const bool on = [] {
    const char* e = getenv("NNC_CUDA_CONV_PAIR");
    return !(e && e[0] == '0');
  }();
  return on;
}

// Whether the paired kernel may split tiles along K (stream-K) when whole
// tiles fill the last wave of pairs badly; NNC_CUDA_CONV_STREAMK=0 turns it
// off (for comparison).
static bool conv_streamk_enabled() {
  static const bool on = [] {
    const char* e = getenv("NNC_CUDA_CONV_STREAMK");
    return !(e && e[0] == '0');
  }();
  return on;
}
// Stream-K needs at least this many k-blocks per tile (shorter reductions
// are HBM-bound, and their partial sums would cost as much as they save) and
// this many iterations per cluster.
constexpr int kStreamKMinKBlocks = 16, kStreamKMinShare = 8;

template <int BN_, int STAGES>
bool launch_conv_pair(ConvArgs g, const float* w0, const char* op, bool streamk_ok) {
  using Cfg = ConvPairCfg<BN_, STAGES>;
  constexpr int BN = Cfg::BN;
  const int Kpad = g.kblocks * BK;
  CUtensorMap tw, tx;
  // Weights: each CTA loads BN / 2 rows of the pair's BN-row tile.
  const uint64_t dims[2] = {(uint64_t)Kpad, (uint64_t)g.Cout};
  const uint64_t strides[1] = {(uint64_t)Kpad * 4};
  const uint32_t box[2] = {BK, BN / 2};
  if (!encode_tmap_f32(&tw, w0, 2, dims, strides, box, nullptr, op)) return false;
  const uint64_t xd[4] = {(uint64_t)g.C4, (uint64_t)g.W, (uint64_t)g.H, (uint64_t)g.N};
  const uint64_t xs[3] = {(uint64_t)g.C4 * 4, (uint64_t)g.W * g.C4 * 4,
                          (uint64_t)g.H * g.W * g.C4 * 4};
  const int lower = -g.ph, upper = (g.OH - 1) * g.sh - g.ph - (g.H - 1);
  if (!encode_tmap_im2col_f32(&tx, g.x_hi, xd, xs, lower, upper, 32, BM, g.sh, true, op))
    return false;
  g.n_tiles = (int)cdiv(g.Cout, BN);
  g.m_tiles = (int)cdiv(g.M, 2 * BM);
  g.tiles = (int64_t)g.m_tiles * g.n_tiles;
  g.direct_epi = direct_epilogue() ? 1 : 0;
  auto kern = conv_tc2_kernel<BN_, STAGES, false>;
  auto kern_sk = conv_tc2_kernel<BN_, STAGES, true>;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kPairThreads, 1, 1);
  cfg.dynamicSmemBytes = Cfg::SMEM;
  cfg.stream = ctx().stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // Per device: the shared-memory opt-in, then how many pairs fit at once.
  static bool attr_set[64] = {};
  static int max_pairs[64] = {};
  if (!attr_set[ctx().device]) {
    if (!check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)Cfg::SMEM),
                    op, "cudaFuncSetAttribute") ||
        !check_cuda(cudaFuncSetAttribute(kern_sk, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)Cfg::SMEM),
                    op, "cudaFuncSetAttribute"))
      return false;
    // Both instances: the stream-K one must fit as many pairs as it is given.
    int n = 0, n_sk = 0;
    cfg.gridDim = dim3(2 * (sm_count() / 2), 1, 1);
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0 ||
        cudaOccupancyMaxActiveClusters(&n_sk, kern_sk, &cfg) != cudaSuccess || n_sk <= 0) {
      cudaGetLastError();
      n = n_sk = sm_count() / 2;
    }
    max_pairs[ctx().device] = n < n_sk ? n : n_sk;
    attr_set[ctx().device] = true;
  }
  const int64_t P = max_pairs[ctx().device];
  int64_t pairs = g.tiles < P ? g.tiles : P;
  // Stream-K when whole tiles would fill the last wave under 90%: the last
  // full wave and the remainder are split into equal shares of k-blocks
  // over all P pairs (every pair is resident at once: P is the occupancy
  // query's count).
  const int64_t waves = cdiv(g.tiles, P);
  // Stride-1 windows only: measured on the ResNet shapes at 128 images,
  // stream-K took stage-3/4 3 x 3 stride-1 convs from 67.6 / 63.5 us to
  // 61.4 / 59.4 but the stride-2 ones from 57.3 / 38.9 us to 61.4 / 43.0.
  if (streamk_ok && conv_streamk_enabled() && g.kblocks >= kStreamKMinKBlocks && g.sh == 1 &&
      g.sw == 1 && g.tiles < waves * P && 10 * g.tiles < 9 * waves * P) {
    const int64_t dp_end = waves >= 2 ? (waves - 2) * P : 0;
    const int64_t iters = (g.tiles - dp_end) * g.kblocks;
    unsigned* count = nullptr;
    float* part = nullptr;
    if (iters >= kStreamKMinShare * P &&
        streamk_scratch((int)P, (size_t)2 * BM * 256 * sizeof(float), &count, &part)) {
      g.sk_dp_tiles = dp_end;
      g.sk_q = iters / P;
      g.sk_r = iters % P;
      g.sk_part = part;
      g.sk_count = count;
      pairs = P;
    }
  }
  cfg.gridDim = dim3((unsigned)(2 * pairs), 1, 1);
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see pdl_trigger
  attr[1].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.numAttrs = 2;
  if (!check_cuda(cudaLaunchKernelEx(&cfg, g.sk_q ? kern_sk : kern, tw, tx, g), op,
                  "cudaLaunchKernelEx"))
    return false;
  return check_launch(op);
}

// Whether a halo call's epilogue takes the direct path (store_tile's
// `direct`, decided the same way in the kernel): channels-last output, C_out
// a multiple of 32, 16-byte aligned output and residual, and a window of
// several taps (a 1 x 1 window's short MMAs leave the shared-memory port to
// the staged path, whose full-line stores measured faster there).
static bool halo_direct(const ConvArgs& g) {
  return direct_epilogue() && g.out_nhwc && perm_rows(g.Cout) &&
         (g.KH * g.KW > 1 || direct_epilogue_mode() == 2) &&
         (((uintptr_t)g.out) & 15) == 0 && (!g.residual || (((uintptr_t)g.residual) & 15) == 0);
}

// Whether halo calls run on CTA pairs (the default); NNC_CUDA_CONV_HALO_PAIR=0
// selects the single-CTA kernel (for comparison).
static bool halo_pair_enabled() {
  static const bool on = [] {
    const char* e = getenv("NNC_CUDA_CONV_HALO_PAIR");
    return !(e && e[0] == '0');
  }();
  return on;
}

// NNC_CUDA_CONV_SMALL_TC=0 keeps few-channel convs on the CUDA-core kernels.
static bool small_tc_enabled() {
  static const bool on = [] {
    const char* e = getenv("NNC_CUDA_CONV_SMALL_TC");
    return !(e && e[0] == '0');
  }();
  return on;
}

template <int KB, bool VEC2>
bool launch_small_tc(const ConvArgs& g, const SmallTcTable& tab, const float* w, int src_mode,
                     int src_c4, int src_kpad, const char* op) {
  using Cfg = SmallTcCfg<KB>;
  auto kern = conv_small_tc_kernel<KB, VEC2>;
  static bool attr_set[64] = {};
  static int per_sm[64] = {};
  if (!attr_set[ctx().device]) {
    if (!check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)Cfg::SMEM),
                    op, "cudaFuncSetAttribute"))
      return false;
    // CTAs an SM holds by shared memory, registers and TMEM (32 of its 512
    // columns each). The grid is sized from these rather than from the
    // occupancy query, which gave one CTA per SM for this kernel; a CTA that
    // does not fit yet only starts when another ends, since CTAs never wait
    // on one another.
    cudaFuncAttributes fa{};
    if (!check_cuda(cudaFuncGetAttributes(&fa, kern), op, "cudaFuncGetAttributes")) return false;
    const int by_smem = (int)((228u * 1024u) / (Cfg::SMEM + 1024u));
    const int by_regs = 65536 / (Cfg::THREADS * (fa.numRegs > 0 ? fa.numRegs : 255));
    int r = by_smem < by_regs ? by_smem : by_regs;
    r = r < 16 ? r : 16;
    per_sm[ctx().device] = r > 0 ? r : 1;
    attr_set[ctx().device] = true;
  }
  const int64_t tiles = cdiv(g.M, BM), cap = (int64_t)sm_count() * per_sm[ctx().device];
  const int grid = (int)(tiles < cap ? tiles : cap);
  ConvArgs a = g;
  a.err = device_error_word();
  kern<<<grid, Cfg::THREADS, Cfg::SMEM, ctx().stream>>>(a, tab, w, src_mode, src_c4, src_kpad);
  return check_launch(op);
}

// Few-channel conv on the tensor-core tile kernel: builds the per-k tables
// (channel pairs adjacent for a channels-last input with an even channel
// count) and picks the instance by k-blocks.
void launch_small_tc_conv(const ConvArgs& g, int C, bool in_nhwc, const float* w, int src_mode,
                          int src_c4, int src_kpad, const char* op) {
  SmallTcTable tab;
  const int KHW = g.KH * g.KW;
  const bool vec2 = in_nhwc && C % 2 == 0 && ((uintptr_t)g.x_hi & 7u) == 0;
  for (int k = 0; k < kSmallTcMaxK; ++k) {
    tab.off[k] = 0;
    tab.bit[k] = 0;
    if (k >= g.K) continue;
    const int c = vec2 ? k % C : k / KHW, t = vec2 ? k / C : k % KHW;
    const int kh = t / g.KW, kw = t - kh * g.KW;
    tab.off[k] = (int)(c * g.xs_c + kh * g.xs_h + kw * g.xs_w);
    tab.bit[k] = 1u << t;
  }
  tab.ohw = fast_div((unsigned)(g.OH * g.OW));
  tab.ow = fast_div((unsigned)g.OW);
  tab.stage = g.out_nhwc && aligned16(g.out) && (!g.residual || aligned16(g.residual));
  const int kb = (int)cdiv(g.K, 32);
  if (kb <= 1)
    vec2 ? launch_small_tc<1, true>(g, tab, w, src_mode, src_c4, src_kpad, op)
         : launch_small_tc<1, false>(g, tab, w, src_mode, src_c4, src_kpad, op);
  else if (kb <= 2)
    vec2 ? launch_small_tc<2, true>(g, tab, w, src_mode, src_c4, src_kpad, op)
         : launch_small_tc<2, false>(g, tab, w, src_mode, src_c4, src_kpad, op);
  else
    vec2 ? launch_small_tc<5, true>(g, tab, w, src_mode, src_c4, src_kpad, op)
         : launch_small_tc<5, false>(g, tab, w, src_mode, src_c4, src_kpad, op);
}

// ----------------------------------------- row-banded conv on tensor cores ----
// Few-channel convs whose output row fits one MMA (OW C_out <= 256) and whose
// input row (x = iw C + c over W C floats: channels-last, or one channel) is
// contiguous. For window row kh, output row (n, oh) takes input row (n, oh -
// ph + kh) times the banded weight T_kh[x][col], col the output column in the
// output's own order ((ow, co) channels-last, (co, ow) otherwise):
// T_kh[x][col] = w[co][c][kh][iw - ow sw + pw] inside the window, 0 elsewhere.
// A tile is IMGS whole images (IMGS OH <= 128 rows). A = one TMA box of input
// rows (a 32-float k-block of each row, OH rows from kh - ph, IMGS images;
// rows and images outside the tensor read as zeros, which is the vertical
// padding); B = that k-block of T_kh, bulk-copied from the banded weight that
// a small kernel builds per call (rows pre-swizzled). The D rows are the
// tile's output rows with all their columns; they are staged in shared memory
// in the output's layout and leave by bulk copy, since a tile's images are
// one contiguous range of the output in either layout. Warp 0 loads, warp 1
// issues the MMAs into two TMEM accumulators, warps 2-17 drain them (bias,
// residual, activation). The tensor cores do ~W C / (C KW) times the useful
// work, which is cheap next to building im2col rows for a few channels.
constexpr int kRowBandEpiWarps = 16;  // four per TMEM lane quadrant, splitting the columns
constexpr int kRowBandThreads = 64 + 32 * kRowBandEpiWarps;
__device__ __forceinline__ void rowband_epi_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(32 * kRowBandEpiWarps) : "memory");
}

struct RowBandArgs {
  const float* band;   // [KH][kb][n_pad][32] pre-swizzled banded weight
  int imgs, nimg;      // images per tile, images in all
  int kb;              // 32-float k-blocks of an input row
  int n_cols, n_pad;   // output columns (OW C_out), rounded up to 16
  int stages;          // load ring depth
  int nchw;            // output column order (co, ow) instead of (ow, co)
  int vec4;            // channels-last with OW C_out a multiple of 4 (float4 staging)
  int row_stride;      // elements between output rows oh, oh + 1 of an image
  int acc_stride;      // TMEM columns between the two accumulators (n_pad rounded up to 32)
  int tmem_cols;       // power of two >= 2 acc_stride
  uint32_t a_bytes, b_bytes, stage_bytes;  // box bytes, n_pad x 128, 16 KB + b_bytes
  uint32_t img_elems;  // C_out OH OW
  uint32_t img_stride; // staged elements per image: img_elems, padded against bank conflicts
  uint32_t out_off, col_off, bar_off;      // shared-memory layout
};

__global__ void __launch_bounds__(kRowBandThreads, 1)
    conv_rowband_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ ConvArgs g,
                        const __grid_constant__ RowBandArgs rb) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  float* obuf = reinterpret_cast<float*>(smem + rb.out_off);
  int* colpart = reinterpret_cast<int*>(smem + rb.col_off);  // column -> offset in an image
  float* biasc = reinterpret_cast<float*>(colpart + rb.n_pad);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + rb.bar_off);
  uint64_t* empty = full + rb.stages;
  uint64_t* tfull = empty + rb.stages;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int OH = g.OH, OW = g.OW, Cout = g.Cout;

  for (int n = threadIdx.x; n < rb.n_pad; n += kRowBandThreads) {
    int cp = 0;
    float bv = 0.0f;
    if (n < rb.n_cols) {
      const int co = rb.nchw ? n / OW : n % Cout, ow = rb.nchw ? n % OW : n / Cout;
      cp = rb.nchw ? co * OH * OW + ow : n;
      if (g.bias) bv = __ldg(g.bias + co);
    }
    colpart[n] = cp;
    biasc[n] = bv;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < rb.stages; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      tc::mbar_init(&tfull[a], 1);
      tc::mbar_init(&tempty[a], kRowBandEpiWarps);
    }
    tc::fence_barrier_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, (uint32_t)rb.tmem_cols);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int tiles = (rb.nimg + rb.imgs - 1) / rb.imgs;

  if (warp == 0) {
    if (lane == 0) {
      tc::prefetch_tmap(&tmX);
      int s = 0;
      uint32_t ph = 0, armed = 0, armed_ph = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x)
        for (int kh = 0; kh < g.KH && ok; ++kh)
          for (int kb = 0; kb < rb.kb; ++kb) {
            if (!tc::mbar_wait(&empty[s], ph ^ 1, g.err)) {
              ok = false;
              break;
            }
            uint8_t* st = smem + s * rb.stage_bytes;
            tc::mbar_arrive_expect_tx(&full[s], rb.a_bytes + rb.b_bytes);
            tc::tma_load_3d(st, &tmX, &full[s], kb * 32, kh - g.ph, tile * rb.imgs);
            tc::bulk_load(st + 16384, rb.band + (size_t)(kh * rb.kb + kb) * rb.n_pad * 32, rb.b_bytes,
                          &full[s]);
            armed |= 1u << s;
            armed_ph = (armed_ph & ~(1u << s)) | (ph << s);
            if (++s == rb.stages) {
              s = 0;
              ph ^= 1;
            }
          }
      // Copies still in flight (only after a wait gave up) land before exit.
      for (int q = 0; q < rb.stages; ++q)
        if ((armed >> q) & 1) tc::mbar_wait(&full[q], (armed_ph >> q) & 1, g.err);
    }
  } else if (warp == 1) {
    const uint32_t idesc = tc::idesc_tf32(BM, rb.n_pad);
    int s = 0, acc = 0;
    uint32_t ph = 0, aph = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
      ok = tc::mbar_wait_warp(&tempty[acc], aph ^ 1, g.err);
      tc::tc_fence_after();
      const int steps = g.KH * rb.kb;
      for (int step = 0; step < steps && ok; ++step) {
        ok = tc::mbar_wait_warp(&full[s], ph, g.err);
        tc::tc_fence_after();
        if (ok && tc::elect_one()) {
          const uint32_t a0 = tc::smem_u32(smem + s * rb.stage_bytes), b0 = a0 + 16384;
#pragma unroll
          for (int k = 0; k < 4; ++k)
            tc::mma_tf32(tmem_base + acc * rb.acc_stride, tc::desc_kmajor_sw128(a0 + k * 32),
                         tc::desc_kmajor_sw128(b0 + k * 32), idesc, (step | k) != 0);
          tc::mma_commit(&empty[s]);
        }
        __syncwarp();
        if (++s == rb.stages) {
          s = 0;
          ph ^= 1;
        }
      }
      if (ok && tc::elect_one()) tc::mma_commit(&tfull[acc]);
      __syncwarp();
      acc ^= 1;
      if (acc == 0) aph ^= 1;
    }
  } else {
    const int quarter = warp & 3, part = (warp - 2) >> 2;  // chunks part, part + 4, ...
    // Channels-last outputs: each TMEM lane quadrant's 32 rows are one
    // contiguous range of the output, stored by the quadrant's own leader
    // once its four warps are done (no tile-wide barrier). NCHW outputs: one
    // leader stores whole images after all sixteen warps.
    const bool by_quadrant = !rb.nchw;
    const bool leader = by_quadrant ? (lane == 0 && part == 0) : threadIdx.x == 64;
    auto quadrant_sync = [&]() {  // named barriers 2-5: the four warps of a quadrant
      switch (quarter) {
        case 0: asm volatile("bar.sync 2, 128;" ::: "memory"); break;
        case 1: asm volatile("bar.sync 3, 128;" ::: "memory"); break;
        case 2: asm volatile("bar.sync 4, 128;" ::: "memory"); break;
        default: asm volatile("bar.sync 5, 128;" ::: "memory"); break;
      }
    };
    const bool add = g.act == kActAddRelu;
    const bool relu = add || g.act == kActRelu, sig = g.act == kActSigmoid;
    int acc = 0;
    uint32_t aph = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
      ok = ok && tc::mbar_wait_warp(&tfull[acc], aph, g.err);
      tc::tc_fence_after();
      if (leader) tc::bulk_wait_group_read<0>();  // the last tile's copy has read obuf
      if (by_quadrant)
        quadrant_sync();
      else
        rowband_epi_sync();
      const int img0 = tile * rb.imgs;
      const int nim = min(rb.imgs, rb.nimg - img0);
      const int r = quarter * 32 + lane;
      const bool live = ok && r < nim * OH;
      const int img = r / OH, oh = r - img * OH;
      const int rowpart = img * (int)rb.img_stride + oh * rb.row_stride;  // in the staging buffer
      const float* res =
          add ? g.residual + (size_t)(img0 + img) * rb.img_elems + oh * rb.row_stride : nullptr;
      // Columns of chunk c (16 from TMEM): bias, residual, activation, into
      // the staging buffer.
      auto drain = [&](int c, const uint32_t(&v)[16]) {
        if (live && rb.vec4) {
          // Channels-last, OW C_out a multiple of 4: four columns per store.
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int n = c * 16 + q * 4;
            if (n < rb.n_cols) {
              float o[4] = {__uint_as_float(v[4 * q]), __uint_as_float(v[4 * q + 1]),
                            __uint_as_float(v[4 * q + 2]), __uint_as_float(v[4 * q + 3])};
              if (g.bias) {
                const float4 b = *reinterpret_cast<const float4*>(biasc + n);
                o[0] = __fadd_rn(o[0], b.x);
                o[1] = __fadd_rn(o[1], b.y);
                o[2] = __fadd_rn(o[2], b.z);
                o[3] = __fadd_rn(o[3], b.w);
              }
              if (add) {
                const float4 rv = __ldg(reinterpret_cast<const float4*>(res + n));
                o[0] = __fadd_rn(o[0], rv.x);
                o[1] = __fadd_rn(o[1], rv.y);
                o[2] = __fadd_rn(o[2], rv.z);
                o[3] = __fadd_rn(o[3], rv.w);
              }
              if (sig) {
#pragma unroll
                for (int e = 0; e < 4; ++e) o[e] = activate(o[e], kActSigmoid);
              } else if (relu) {
#pragma unroll
                for (int e = 0; e < 4; ++e) o[e] = o[e] > 0.0f ? o[e] : 0.0f;
              }
              *reinterpret_cast<float4*>(obuf + rowpart + n) = make_float4(o[0], o[1], o[2], o[3]);
            }
          }
        } else if (live) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int n = c * 16 + j;
            if (n < rb.n_cols) {
              float o = __uint_as_float(v[j]);
              if (g.bias) o = __fadd_rn(o, biasc[n]);
              if (add) o = __fadd_rn(o, __ldg(res + colpart[n]));
              if (sig)
                o = activate(o, kActSigmoid);
              else if (relu)
                o = o > 0.0f ? o : 0.0f;
              obuf[rowpart + colpart[n]] = o;
            }
          }
        }
      };
      // This warp's chunks (every fourth one) three at a time: the TMEM loads
      // are issued together and waited for once.
      const int nch = rb.n_pad / 16;
      const uint32_t tbase = tmem_base + (uint32_t)(acc * rb.acc_stride) + ((uint32_t)(quarter * 32) << 16);
      for (int c0 = part; c0 < nch; c0 += 12) {
        uint32_t v[3][16];
#pragma unroll
        for (int u = 0; u < 3; ++u)
          if (c0 + 4 * u < nch) tc::tmem_ld16(tbase + (uint32_t)((c0 + 4 * u) * 16), v[u]);
        tc::tmem_ld_wait();
#pragma unroll
        for (int u = 0; u < 3; ++u)
          if (c0 + 4 * u < nch) drain(c0 + 4 * u, v[u]);
      }
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&tempty[acc]);
      tc::fence_proxy_async_smem();  // obuf -> the bulk copy's reads
      if (by_quadrant) {
        quadrant_sync();
        const int r0 = quarter * 32, r1 = min(r0 + 32, nim * OH);
        if (leader && ok && r1 > r0) {
          tc::bulk_store(g.out + ((size_t)img0 * OH + r0) * rb.n_cols, obuf + (size_t)r0 * rb.n_cols,
                         (uint32_t)(r1 - r0) * (uint32_t)rb.n_cols * 4u);
          tc::bulk_commit_group();
        }
      } else {
        rowband_epi_sync();
      }
      if (!by_quadrant && leader && ok) {
        if (rb.img_stride == rb.img_elems) {
          tc::bulk_store(g.out + (size_t)img0 * rb.img_elems, obuf, (uint32_t)nim * rb.img_elems * 4u);
        } else {
          for (int i = 0; i < nim; ++i)
            tc::bulk_store(g.out + (size_t)(img0 + i) * rb.img_elems, obuf + (size_t)i * rb.img_stride,
                           rb.img_elems * 4u);
        }
        tc::bulk_commit_group();
      }
      acc ^= 1;
      if (acc == 0) aph ^= 1;
    }
    if (leader) tc::bulk_wait_group<0>();
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem_base, (uint32_t)rb.tmem_cols);
  }
}

// Builds the banded weight of conv_rowband_kernel from an OIHW or prepacked
// weight: element (kh, kb, col, k) at [kh][kb][col][k] with the row's 16-byte
// chunks in the 128-byte swizzle order (chunk j of row col at j ^ (col & 7)).
__global__ void rowband_weight_kernel(ConvArgs g, RowBandArgs rb, float* band, const float* __restrict__ w,
                                      int src_mode, int src_c4, int src_kpad, int C) {
  const int64_t total = (int64_t)g.KH * rb.kb * rb.n_pad * 32;
  const int KHW = g.KH * g.KW;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int kk = (int)(idx & 31);
    int64_t rest = idx >> 5;
    const int n = (int)(rest % rb.n_pad);
    rest /= rb.n_pad;
    const int kb = (int)(rest % rb.kb), kh = (int)(rest / rb.kb);
    const int x = kb * 32 + kk;
    float v = 0.0f;
    if (n < rb.n_cols && x < g.W * C) {
      const int iw = x / C, c = x - iw * C;
      const int co = rb.nchw ? n / g.OW : n % g.Cout, ow = rb.nchw ? n % g.OW : n / g.Cout;
      const int kw = iw - ow * g.sw + g.pw;
      if (kw >= 0 && kw < g.KW) {
        const int t = kh * g.KW + kw;
        if (src_mode == 0) {
          v = w[(int64_t)co * g.K + c * KHW + t];
        } else {
          const int64_t off = (int64_t)co * src_kpad + (src_mode == 1 ? t * src_c4 + c : c * KHW + t);
          v = __fadd_rn(w[off], w[(int64_t)g.Cout * src_kpad + off]);
        }
      }
    }
    band[(idx >> 5) * 32 + (((kk >> 2) ^ (n & 7)) << 2) + (kk & 3)] = v;
  }
}

template <int BN, int G, int STAGES, int CB, bool POOL, bool STAGED, bool PAIR, bool GATHER>
bool launch_halo_kernel(ConvArgs g, const float* w0, const char* op) {
  using Cfg = HaloCfg<BN, G, STAGES, CB, POOL, STAGED, PAIR, GATHER>;
  static_assert(Cfg::SMEM <= 227 * 1024, "halo instance exceeds the shared memory of a CTA");
  constexpr int kThreads = kHaloThreads + (GATHER ? kGatherThreads : 0);
  const int Kpad = g.K;  // taps x C4, a multiple of CB
  CUtensorMap tw, tx;
  const uint64_t dims[2] = {(uint64_t)Kpad, (uint64_t)g.Cout};
  const uint64_t strides[1] = {(uint64_t)Kpad * 4};
  const uint32_t box[2] = {CB, PAIR ? BN / 2 : BN};
  if (!encode_tmap_f32(&tw, w0, 2, dims, strides, box, nullptr, op, Cfg::ROW)) return false;
  // Input windows: CB channels x (8 + KW - 1) x (32 + KH - 1) pixels of one image.
  const uint64_t xd[4] = {(uint64_t)g.C4, (uint64_t)g.W, (uint64_t)g.H, (uint64_t)g.N};
  const uint64_t xs[3] = {(uint64_t)g.C4 * 4, (uint64_t)g.W * g.C4 * 4,
                          (uint64_t)g.H * g.W * g.C4 * 4};
  // A strided (1 x 1, stride s) window reads every s-th pixel: the box spans
  // s times the pixels it delivers (TMA element strides).
  const uint32_t xbox[4] = {CB, (uint32_t)((kHaloTW + g.KW - 1) * g.sw),
                            (uint32_t)((2 * kHaloTH + g.KH - 1) * g.sh), 1};
  const uint32_t xes[4] = {1, (uint32_t)g.sw, (uint32_t)g.sh, 1};
  if (GATHER)
    memset(&tx, 0, sizeof(tx));  // windows come from the gathering warps
  else if (!encode_tmap_f32(&tx, g.x_hi, 4, xd, xs, xbox, xes, op, Cfg::ROW))
    return false;
  g.tiles_x = (int)cdiv(g.OW, kHaloTW);
  g.tiles_y = (int)cdiv(g.OH, 2 * kHaloTH);
  g.m_tiles = g.N * g.tiles_x * g.tiles_y;
  g.n_tiles = (int)cdiv(g.Cout, BN);
  g.tiles = (int64_t)g.m_tiles * g.n_tiles;
  auto kern = conv_halo_kernel<BN, G, STAGES, CB, POOL, STAGED, PAIR, GATHER>;
  g.direct_epi = halo_direct(g) ? 1 : 0;
  if (!STAGED && !POOL && !g.direct_epi) {
    fail(NNC_CUDA_ERR_INVALID, op, "internal: unstaged halo instance for a staged epilogue");
    return false;
  }
  // POOL: whole images per CTA.
  const int64_t units = POOL ? (int64_t)g.N : (PAIR ? cdiv(g.m_tiles, 2) * g.n_tiles : g.tiles);
  static bool attr_set[64] = {};
  static int max_units[64] = {};
  if (!PAIR) {
    if (!attr_set[ctx().device]) {
      if (!check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)Cfg::SMEM),
                      op, "cudaFuncSetAttribute"))
        return false;
      attr_set[ctx().device] = true;
    }
    const int grid = (int)(units < sm_count() ? units : sm_count());
    launch_pdl(kern, grid, kThreads, Cfg::SMEM, tw, tx, g);
    return check_launch(op);
  }
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = Cfg::SMEM;
  cfg.stream = ctx().stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // Per device: the shared-memory opt-in, then how many pairs fit at once.
  if (!attr_set[ctx().device]) {
    if (!check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)Cfg::SMEM),
                    op, "cudaFuncSetAttribute"))
      return false;
    int n = 0;
    cfg.gridDim = dim3(2 * (sm_count() / 2), 1, 1);
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = sm_count() / 2;
    }
    max_units[ctx().device] = n;
    attr_set[ctx().device] = true;
  }
  const int64_t pairs = units < max_units[ctx().device] ? units : max_units[ctx().device];
  cfg.gridDim = dim3((unsigned)(2 * pairs), 1, 1);
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see pdl_trigger
  attr[1].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.numAttrs = 2;
  if (!check_cuda(cudaLaunchKernelEx(&cfg, kern, tw, tx, g), op, "cudaLaunchKernelEx")) return false;
  return check_launch(op);
}

// The halo kernel for a call: on CTA pairs unless turned off, a lone tile
// would leave the pair's second CTA only a stand-in, or the epilogue pools.
// Measured at batch 1024 (graph replay): ResNet stage-1 3 x 3 convs 474 ->
// 419 us and stage-2 3 x 3 convs 360 -> 338 us on pairs (M = 256 MMAs: each
// SM reads its 128 rows of the window and half of the weight tile, 5 KB per
// N = 64 MMA instead of 6, against the shared-memory port that bounds N <=
// 128); the pooled stem went 1.57 -> 1.76 ms in lockstep pairs, whose MMAs
// wait for both CTAs' heavier epilogues.
// PG, PSTAGES: the weight ring of the CTA-pair instance (taps per stage,
// stages), whose per-tap weight tiles are half as large.
template <int BN, int G, int STAGES, int CB, bool POOL = false, bool STAGED = true,
          bool GATHER = false, int PG = G, int PSTAGES = STAGES>
bool launch_halo(ConvArgs g, const float* w0, const char* op) {
  const int64_t m_tiles = (int64_t)g.N * cdiv(g.OW, kHaloTW) * cdiv(g.OH, 2 * kHaloTH);
  if constexpr (!POOL && !GATHER) {
    if (halo_pair_enabled() && m_tiles >= 2)
      return launch_halo_kernel<BN, PG, PSTAGES, CB, POOL, STAGED, true, false>(g, w0, op);
  }
  return launch_halo_kernel<BN, G, STAGES, CB, POOL, STAGED, false, GATHER>(g, w0, op);
}

// Whether the pooled stem builds its space-to-depth windows in the conv
// kernel (the default); NNC_CUDA_STEM_GATHER=0 runs the separate
// space-to-depth pass instead (for comparison).
static bool stem_gather_enabled() {
  static const bool on = [] {
    const char* e = getenv("NNC_CUDA_STEM_GATHER");
    return !(e && e[0] == '0');
  }();
  return on;
}

// Whether the halo kernel serves a call: stride 1 with windows of at most
// 4 x 4, or a 1 x 1 window with stride 2 (a strided window load), 32-channel
// blocks, TF32, and 8 x 32 output tiles that waste at most ~35% of their rows
// on the image's ragged edge. C_out above 128 runs as several 128-channel
// tiles.
// NNC_CUDA_CONV_HALO=0 in the environment turns the path off (the im2col
// kernel then serves these calls).
bool halo_eligible(int C4, int Cout, int KH, int KW, int sh, int sw, int ph, int pw, int OH, int OW,
                   bool split, int cb = BK) {
  static const bool enabled = [] {
    const char* e = getenv("NNC_CUDA_CONV_HALO");
    return !(e && e[0] == '0');
  }();
  // Stride-2 1 x 1 windows (the projections) read a strided window per tile;
  // above 64 output channels the im2col route's CTA pairs are faster (the
  // ResNet stage-2 projection at batch 1024: 138 against 193 us).
  const bool strided_1x1 = KH == 1 && KW == 1 && sh == 2 && sw == 2 && Cout <= 64;
  if (!enabled || split || C4 % cb != 0) return false;
  if (!(sh == 1 && sw == 1) && !strided_1x1) return false;
  if (KH > kHaloMaxK || KW > kHaloMaxK || ph < 0 || pw < 0 || ph >= KH || pw >= KW) return false;
  const int64_t covered =
      cdiv((int64_t)OW, kHaloTW) * kHaloTW * cdiv((int64_t)OH, 2 * kHaloTH) * 2 * kHaloTH;
  return covered * 100 <= (int64_t)OH * OW * 135;
}

bool conv_f32(const Tensor* t, const char* op, const char* name) {
  if (!valid_tensor(t, op, name)) return false;
  if (elem_type(t) != NNC_DTYPE_FLOAT32) {
    fail(NNC_CUDA_ERR_UNSUPPORTED, op, "%s: only float32 is supported", name);
    return false;
  }
  return true;
}

// Fixed-size device scratch of nnc_conv_static_scratch: the converted input
// planes and packed weights of one call live here instead of in the
// runtime's growable workspace. File-scope, so every device that loads this
// module holds kStaticScratchBytes until the process exits; all calls share
// it, and it keeps the previous call's contents.
constexpr size_t kStaticScratchBytes = size_t(16) << 20;  // 16 MiB
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

struct StaticScratch {
  float* ptr;
  size_t bytes;
};

// Address of g_static_scratch on the current device, resolved once per device
// (the first nnc_conv_static_scratch call on that device, with it current).
// Returns false with the thread's status set when it cannot be resolved.
bool static_scratch_on_device(StaticScratch* out, const char* op) {
  constexpr int kDevices = 64;
  static std::mutex mu;
  static float* ptrs[kDevices] = {};
  const int dev = ctx().device;
  if (dev < 0 || dev >= kDevices) {
    fail(NNC_CUDA_ERR_INVALID, op, "device %d is outside the %d devices this library tracks", dev,
         kDevices);
    return false;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!ptrs[dev]) {
    float* ptr = nullptr;
    if (!check_cuda(cudaGetSymbolAddress((void**)&ptr, g_static_scratch), op,
                    "cudaGetSymbolAddress(g_static_scratch)"))
      return false;
    ptrs[dev] = ptr;
  }
  out->ptr = ptrs[dev];
  out->bytes = kStaticScratchBytes;
  return true;
}

// Stride-2 convolutions over at most 8 channels run as stride-1
// convolutions over the space-to-depth input (4 C channels, padded to 32):
// tap kh of the original window maps to s2d tap kh2 = (kh - ph - dy) / 2 +
// pad_h for the pixel-row parity dy. Returns false when the s2d window would
// exceed the halo kernel's 4 x 4.
struct S2dPlan {
  int KH2, KW2, pad_h, pad_w;
};
bool s2d_plan(int C, int KH, int KW, int sh, int sw, int ph, int pw, S2dPlan* p) {
  if (sh != 2 || sw != 2 || C < 1 || 4 * C > BK || ph < 0 || pw < 0) return false;
  auto floor_div2 = [](int a) { return a >= 0 ? a / 2 : -((-a + 1) / 2); };
  const int a_min_h = -((ph + 1) / 2), a_max_h = floor_div2(KH - 1 - ph);
  const int a_min_w = -((pw + 1) / 2), a_max_w = floor_div2(KW - 1 - pw);
  p->KH2 = a_max_h - a_min_h + 1;
  p->KW2 = a_max_w - a_min_w + 1;
  p->pad_h = -a_min_h;
  p->pad_w = -a_min_w;
  return p->KH2 >= 1 && p->KW2 >= 1 && p->KH2 <= kHaloMaxK && p->KW2 <= kHaloMaxK;
}

// NNC_CUDA_CONV_ROWBAND=0 keeps these convs off the row-banded kernel.
static bool rowband_enabled() {
  static const bool on = [] {
    const char* e = getenv("NNC_CUDA_CONV_ROWBAND");
    return !(e && e[0] == '0');
  }();
  return on;
}

// Shape of the row-banded kernel for a call (input rows contiguous: one
// channel or channels-last); false when the call does not fit it: stride 1
// down the rows, input rows of 32 to 256 floats (a multiple of 4), at most 128
// output rows per image, at most 256 output columns (OW C_out), images of a
// multiple of 4 output elements, and a load ring of at least two stages beside
// a tile's staged output in shared memory.
static bool rowband_plan(const ConvArgs& g, int C, RowBandArgs* rb, size_t* smem, size_t* band_bytes) {
  const int64_t L = (int64_t)g.W * C;
  const int64_t n_cols = (int64_t)g.OW * g.Cout;
  if (g.sh != 1 || L < 32 || L > 256 || L % 4 != 0 || g.OH > 128 || g.OH > g.H || n_cols > 256 ||
      (n_cols * g.OH) % 4 != 0)
    return false;
  RowBandArgs r{};
  r.imgs = (int)(128 / g.OH < g.N ? 128 / g.OH : g.N);
  r.nimg = g.N;
  r.kb = (int)cdiv(L, 32);
  r.n_cols = (int)n_cols;
  r.n_pad = (int)cdiv(n_cols, 16) * 16;
  r.nchw = g.out_nhwc ? 0 : 1;
  r.vec4 = g.out_nhwc && n_cols % 4 == 0;
  r.row_stride = g.out_nhwc ? (int)n_cols : g.OW;
  r.acc_stride = (int)cdiv(r.n_pad, 32) * 32;
  r.tmem_cols = 32;
  while (r.tmem_cols < 2 * r.acc_stride) r.tmem_cols *= 2;
  r.a_bytes = (uint32_t)(128 * g.OH * r.imgs);
  r.b_bytes = (uint32_t)r.n_pad * 128;
  r.stage_bytes = 16384 + r.b_bytes;
  r.img_elems = (uint32_t)(n_cols * g.OH);
  // NCHW staging writes: the lanes of a warp hold consecutive output rows,
  // OW apart within an image and img_stride apart across images. Pad the
  // image stride (by a multiple of 4 floats, keeping each image's copy
  // 16-byte aligned) to the value that spreads those rows over the most
  // shared-memory banks.
  r.img_stride = r.img_elems;
  if (r.nchw) {
    int best = 1 << 30;
    for (uint32_t pad = 0; pad < 32; pad += 4) {
      int cost = 0;
      for (int q = 0; q < 4; ++q) {
        int hits[32] = {}, worst = 0;
        for (int row = 32 * q; row < 32 * q + 32 && row < r.imgs * g.OH; ++row) {
          const int img = row / g.OH, oh = row - img * g.OH;
          const int b = (int)(((int64_t)img * (r.img_elems + pad) + (int64_t)oh * g.OW) & 31);
          worst = ++hits[b] > worst ? hits[b] : worst;
        }
        cost += worst;
      }
      if (cost < best) {
        best = cost;
        r.img_stride = r.img_elems + pad;
      }
    }
  }
  const uint32_t out_bytes = (uint32_t)cdiv((int64_t)r.imgs * r.img_stride * 4, 1024) * 1024;
  const uint32_t col_bytes = (uint32_t)r.n_pad * 8;  // column offsets and biases
  const uint32_t fixed_bytes = out_bytes + col_bytes + 8 * (2 * 8 + 4) + 16 + 1024;
  const int64_t stages = ((int64_t)227 * 1024 - fixed_bytes) / r.stage_bytes;
  if (stages < 2) return false;
  r.stages = (int)(stages < 8 ? stages : 8);
  r.out_off = (uint32_t)r.stages * r.stage_bytes;
  r.col_off = r.out_off + out_bytes;
  r.bar_off = r.col_off + col_bytes;
  *smem = (size_t)r.bar_off + 8 * (2 * r.stages + 4) + 16 + 1024;
  *band_bytes = (size_t)g.KH * r.kb * r.n_pad * 128;
  *rb = r;
  return true;
}

// Builds the banded weight (in the workspace, or the fixed scratch) and runs
// the row-banded kernel on a persistent grid.
static void launch_rowband(ConvArgs g, int C, const RowBandArgs& plan, size_t smem, size_t band_bytes,
                           const float* w, int src_mode, int src_c4, int src_kpad,
                           const StaticScratch* fixed, const char* op) {
  float* band = nullptr;
  if (fixed) {
    if (band_bytes > fixed->bytes) {
      fail(NNC_CUDA_ERR_INVALID, op, "needs %zu bytes of scratch; the static scratch holds %zu",
           band_bytes, fixed->bytes);
      return;
    }
    band = fixed->ptr;
  } else {
    band = (float*)workspace(band_bytes, op);
    if (!band) return;
  }
  RowBandArgs rb = plan;
  rb.band = band;
  cudaStream_t st = ctx().stream;
  const int64_t total = (int64_t)band_bytes / 4;
  rowband_weight_kernel<<<grid_for(total, 256), 256, 0, st>>>(g, rb, band, w, src_mode, src_c4, src_kpad, C);
  if (!check_launch(op)) return;
  CUtensorMap tm;
  const uint64_t L = (uint64_t)g.W * C;
  const uint64_t dims[3] = {L, (uint64_t)g.H, (uint64_t)g.N};
  const uint64_t strides[2] = {L * 4, L * g.H * 4};
  const uint32_t box[3] = {32, (uint32_t)g.OH, (uint32_t)rb.imgs};
  if (!encode_tmap_f32(&tm, g.x_hi, 3, dims, strides, box, nullptr, op)) return;
  static bool attr_set[64] = {};
  if (!attr_set[ctx().device]) {
    if (!check_cuda(cudaFuncSetAttribute(conv_rowband_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         227 * 1024),
                    op, "cudaFuncSetAttribute"))
      return;
    attr_set[ctx().device] = true;
  }
  const int tiles = (int)cdiv(g.N, rb.imgs);
  const int grid = tiles < sm_count() ? tiles : sm_count();
  g.err = device_error_word();
  conv_rowband_kernel<<<grid, kRowBandThreads, smem, st>>>(tm, g, rb);
  check_launch(op);
}

// fixed == nullptr: scratch comes from the runtime workspace (which may grow
// with cudaMallocAsync); otherwise from *fixed, and a call that needs more
// than it holds is rejected before any work is queued.
// Max pooling applied to the conv result (nnc_conv_relu_maxpool): the conv's
// own output extent and the pool window, stride and top/left pad.
struct PoolSpec {
  int conv_h, conv_w, kh, kw, sh, sw, ph, pw;
};

void conv_impl(Tensor* input, Tensor* weight, Tensor* bias, Tensor* residual, Tensor* output,
               int KH, int KW, int sh, int sw, int ph, int pw, int act, const char* op,
               const StaticScratch* fixed = nullptr, const PoolSpec* pool = nullptr) {
  if (!conv_f32(input, op, "input") || !conv_f32(weight, op, "weight") ||
      !conv_f32(output, op, "output"))
    return;
  if (bias && !conv_f32(bias, op, "bias")) return;
  if (residual && !conv_f32(residual, op, "residual")) return;
  if (input->ndim != 4 || weight->ndim != 4 || output->ndim != 4) {
    fail(NNC_CUDA_ERR_INVALID, op, "expected 4-D tensors");
    return;
  }
  trace_io(tensor_bytes(input) + tensor_bytes(weight) + tensor_bytes(bias) + tensor_bytes(residual),
           tensor_bytes(output));
  const int N = (int)input->shape[0], C = (int)input->shape[1], H = (int)input->shape[2],
            W = (int)input->shape[3];
  const int Cout = (int)weight->shape[0];
  // With a fused pool the output tensor is the pooled one; the conv extent
  // comes with the pool spec.
  const int OH = pool ? pool->conv_h : (int)output->shape[2];
  const int OW = pool ? pool->conv_w : (int)output->shape[3];
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
  if (pool && (residual || pool->kh <= 0 || pool->kw <= 0 || pool->sh <= 0 || pool->sw <= 0 ||
               OH <= 0 || OW <= 0)) {
    fail(NNC_CUDA_ERR_INVALID, op, "invalid pooled conv geometry");
    return;
  }
  const int64_t M = (int64_t)N * OH * OW;
  if (M == 0 || Cout == 0) return;
  const bool split = ctx().precision == NNC_CUDA_PRECISION_3XTF32;
  // Few output channels and a short reduction: in TF32 mode with many pixels
  // the tensor-core kernels below (row-banded, else im2col tiles); otherwise
  // the direct CUDA-core kernels (full fp32, so either precision mode).
  if (!pool && Cout <= 16 && (int64_t)C * KH * KW <= kDirectMaxK && (int64_t)C * H * W < (1ll << 31)) {
    const bool packed_w = (tag_of(weight) & NNC_CUDA_TAG_PACKED_CONV) != 0;
    const WeightLayout wl0 = weight_layout(C, KH, KW);
    ConvArgs g{};
    g.N = N;
    g.H = H;
    g.W = W;
    g.OH = OH;
    g.OW = OW;
    g.Cout = Cout;
    g.KH = KH;
    g.KW = KW;
    g.sh = sh;
    g.sw = sw;
    g.ph = ph;
    g.pw = pw;
    g.K = C * KH * KW;
    g.M = M;
    g.x_hi = (const float*)input->data;
    const bool in_nhwc = is_nhwc(input);
    g.xs_n = (int64_t)C * H * W;
    g.xs_c = in_nhwc ? 1 : (int64_t)H * W;
    g.xs_h = in_nhwc ? (int64_t)W * C : W;
    g.xs_w = in_nhwc ? C : 1;
    g.bias = bias ? (const float*)bias->data : nullptr;
    g.residual = residual ? (const float*)residual->data : nullptr;
    g.out = (float*)output->data;
    g.out_nhwc = is_nhwc(output) ? 1 : 0;
    g.act = act;
    const int src_mode = packed_w ? (wl0.element ? 2 : 1) : 0;
    const int grid = (int)(cdiv(M, 128) < (int64_t)sm_count() * 8 ? cdiv(M, 128) : (int64_t)sm_count() * 8);
    const float* wp = (const float*)weight->data;
    cudaStream_t st = ctx().stream;
    // TF32 mode with many pixels: the row-banded tensor-core kernel where
    // input rows are contiguous and an output row fits one MMA, else the
    // im2col tile kernel.
    if (!split && M >= kSmallTcMinM && rowband_enabled() && (C == 1 || in_nhwc) &&
        aligned16(g.x_hi) && aligned16(g.out)) {
      RowBandArgs rb{};
      size_t smem = 0, band_bytes = 0;
      if (rowband_plan(g, (int)C, &rb, &smem, &band_bytes)) {
        launch_rowband(g, (int)C, rb, smem, band_bytes, wp, src_mode, wl0.C4, wl0.Kpad, fixed, op);
        return;
      }
    }
    if (!split && M >= kSmallTcMinM && M + BM < (1ll << 31) && g.K <= kSmallTcMaxK && KH * KW <= 32 &&
        small_tc_enabled()) {
      launch_small_tc_conv(g, (int)C, in_nhwc, wp, src_mode, wl0.C4, wl0.Kpad, op);
      return;
    }
    // Row-blocked kernel for stride-1-wide 3- and 5-wide windows: 4 output
    // pixels per thread, 8 channels per thread (two threads per pixel block
    // above 8 output channels).
    const int cgs = Cout <= 8 ? 1 : 2;
    const int64_t units = (int64_t)N * OH * cdiv(OW, 4) * cgs;
    const int grid4 = (int)(cdiv(units, 128) < (int64_t)sm_count() * 8 ? cdiv(units, 128)
                                                                         : (int64_t)sm_count() * 8);
    if (sw == 1 && (KW == 5 || KW == 3) && units + (int64_t)grid4 * 128 < (1ll << 31)) {
      if (Cout <= 8 && KW == 5)
        conv_direct_row_kernel<8, 1, 5, 4><<<grid4, 128, 0, st>>>(g, wp, src_mode, wl0.C4, wl0.Kpad);
      else if (KW == 5)
        conv_direct_row_kernel<8, 2, 5, 4><<<grid4, 128, 0, st>>>(g, wp, src_mode, wl0.C4, wl0.Kpad);
      else if (Cout <= 8)
        conv_direct_row_kernel<8, 1, 3, 4><<<grid4, 128, 0, st>>>(g, wp, src_mode, wl0.C4, wl0.Kpad);
      else
        conv_direct_row_kernel<8, 2, 3, 4><<<grid4, 128, 0, st>>>(g, wp, src_mode, wl0.C4, wl0.Kpad);
    } else if (Cout <= 8)
      conv_direct_kernel<8><<<grid, 128, 0, ctx().stream>>>(g, (const float*)weight->data, src_mode,
                                                            wl0.C4, wl0.Kpad);
    else
      conv_direct_kernel<16><<<grid, 128, 0, ctx().stream>>>(g, (const float*)weight->data, src_mode,
                                                             wl0.C4, wl0.Kpad);
    check_launch(op);
    return;
  }
  const WeightLayout wl = weight_layout(C, KH, KW);
  const int C4 = wl.C4;
  const int Kpad = wl.Kpad;
  const bool packed = (tag_of(weight) & NNC_CUDA_TAG_PACKED_CONV) != 0;

  // Stride-2 convolutions over few channels: space-to-depth, then the halo
  // kernel (stride 1, 32 channels). Falls through to the general path when
  // the rewritten call is not eligible or its scratch exceeds a fixed scratch.
  S2dPlan s2d;
  const int C2 = 4 * C <= 16 ? 16 : BK;  // stored s2d channels: 64- or 128-byte pixel rows
  // Fused pooling: one channel tile (C_out <= 64), a conv row that fits the
  // row carry, a channels-last pooled output, and stride-2 windows that hold
  // their centre (2 py, 2 px) inside the conv result and reach at most one
  // row/column before and after it.
  const bool pool_fused =
      pool && C2 == 16 && Cout <= 64 && OW <= kPoolMaxOW && is_nhwc(output) && pool->sh == 2 &&
      pool->sw == 2 && pool->ph >= 0 && pool->pw >= 0 && pool->ph <= 1 && pool->pw <= 1 &&
      pool->kh > pool->ph && pool->kw > pool->pw && pool->kh - pool->ph <= 2 &&
      pool->kw - pool->pw <= 2 && 2 * ((int)output->shape[2] - 1) < OH &&
      2 * ((int)output->shape[3] - 1) < OW;
  if (!split && (!pool || pool_fused) && s2d_plan(C, KH, KW, sh, sw, ph, pw, &s2d) &&
      halo_eligible(C2, Cout, s2d.KH2, s2d.KW2, 1, 1, s2d.pad_h, s2d.pad_w, OH, OW, split, C2)) {
    const int H2 = (H + 1) / 2, W2 = (W + 1) / 2;
    // The pooled 3-channel stem gathers its windows in the conv kernel: no
    // space-to-depth copy of the input.
    const bool gather = pool_fused && C == 3 && stem_gather_enabled();
    const int64_t x2 = gather ? 0 : (int64_t)N * H2 * W2 * C2,
                  w2 = (int64_t)Cout * s2d.KH2 * s2d.KW2 * C2;
    const size_t need2 = (size_t)((x2 + 63) / 64 * 64 + w2) * 4 + 256;
    if (!fixed || need2 <= fixed->bytes) {
      float* ws2 = fixed ? fixed->ptr : (float*)workspace(need2, op);
      if (!ws2) return;
      float* xs2 = ws2;
      float* wts2 = ws2 + (x2 + 63) / 64 * 64;
      const bool in_nhwc = is_nhwc(input);
      const int64_t sx_c = in_nhwc ? 1 : (int64_t)H * W, sx_h = in_nhwc ? (int64_t)W * C : W,
                    sx_w = in_nhwc ? C : 1;
      const size_t rows_smem = (size_t)2 * C * W * 4;
      if (gather) {
        // nothing to convert
      } else if (!in_nhwc && rows_smem <= 48 * 1024) {
        const bool vec = W % 4 == 0 && (((uintptr_t)input->data) & 15) == 0;
        const float* xin = (const float*)input->data;
        const int64_t xs_n = (int64_t)H * W * C;
        const unsigned blocks = (unsigned)((int64_t)N * H2);
        if (C2 == 16 && vec)
          launch_pdl(s2d_rows_kernel<16, true>, blocks, 128, rows_smem,
              xin, xs2, C, H, W, H2, W2, xs_n, sx_c, sx_h);
        else if (C2 == 16)
          launch_pdl(s2d_rows_kernel<16, false>, blocks, 128, rows_smem,
              xin, xs2, C, H, W, H2, W2, xs_n, sx_c, sx_h);
        else if (vec)
          launch_pdl(s2d_rows_kernel<BK, true>, blocks, 128, rows_smem,
              xin, xs2, C, H, W, H2, W2, xs_n, sx_c, sx_h);
        else
          launch_pdl(s2d_rows_kernel<BK, false>, blocks, 128, rows_smem,
              xin, xs2, C, H, W, H2, W2, xs_n, sx_c, sx_h);
      } else if (C2 == 16) {
        s2d_input_kernel<16><<<grid_for(x2 / C2, 256, 8), 256, 0, ctx().stream>>>(
            (const float*)input->data, xs2, N, C, H, W, H2, W2, (int64_t)H * W * C, sx_c, sx_h,
            sx_w);
      } else {
        s2d_input_kernel<BK><<<grid_for(x2 / C2, 256, 8), 256, 0, ctx().stream>>>(
            (const float*)input->data, xs2, N, C, H, W, H2, W2, (int64_t)H * W * C, sx_c, sx_h,
            sx_w);
      }
      if (!gather && !check_launch(op)) return;
      const int src_mode = packed ? (wl.element ? 2 : 1) : 0;
      launch_pdl(s2d_weight_kernel, grid_for(w2, 256, 8), 256, 0, (const float*)weight->data, wts2,
                 Cout, C, KH, KW, ph, pw, s2d.KH2, s2d.KW2, s2d.pad_h, s2d.pad_w, src_mode, wl.C4,
                 wl.Kpad, C2);
      if (!check_launch(op)) return;
      ConvArgs g{};
      g.mode = kHalo;
      g.N = N;
      g.H = H2;
      g.W = W2;
      g.C4 = C2;
      g.OH = OH;
      g.OW = OW;
      g.Cout = Cout;
      g.KH = s2d.KH2;
      g.KW = s2d.KW2;
      g.sh = g.sw = 1;
      g.ph = s2d.pad_h;
      g.pw = s2d.pad_w;
      g.K = s2d.KH2 * s2d.KW2 * C2;
      g.kblocks = (int)cdiv(g.K, BK);
      g.M = M;
      g.x_hi = xs2;
      g.bias = bias ? (const float*)bias->data : nullptr;
      g.residual = residual ? (const float*)residual->data : nullptr;
      g.out = (float*)output->data;
      g.out_nhwc = is_nhwc(output) ? 1 : 0;
      g.act = act;
      g.err = device_error_word();
      if (pool_fused) {
        g.pool = 1;
        g.PH = (int)output->shape[2];
        g.PW = (int)output->shape[3];
        g.pkh = pool->kh;
        g.pkw = pool->kw;
        g.psh = pool->sh;
        g.psw = pool->sw;
        g.pph = pool->ph;
        g.ppw = pool->pw;
        if (gather) {
          g.x_hi = nullptr;
          g.src = (const float*)input->data;
          g.src_H = H;
          g.src_W = W;
          g.src_sn = (int64_t)H * W * C;
          g.src_sc = sx_c;
          g.src_sh = sx_h;
          g.src_sw = sx_w;
          // Two weight stages (the 16 resident taps): measured at batch
          // 1024, 1279 us against 1383 with three; the smaller shared
          // allocation leaves L1 room for the gathered rows (a third window
          // slot: 1350; an L2 bulk prefetch of the next tile's rows: 2057).
          launch_halo<64, 8, 2, 16, true, true, true>(g, wts2, op);
        } else {
          launch_halo<64, 8, 3, 16, true>(g, wts2, op);
        }
        return;
      } else if (C2 == 16) {
        if (Cout > 64)
          launch_halo<128, 2, 4, 16>(g, wts2, op);
        else
          launch_halo<64, 8, 3, 16>(g, wts2, op);
      } else {
        if (Cout > 64)
          launch_halo<128, 1, 4, 32>(g, wts2, op);
        else
          launch_halo<64, 3, 3, 32>(g, wts2, op);
      }
      return;
    }
  }
  if (pool) {
    // Composition: the conv into a temporary tensor (the output's layout),
    // then max pooling into the output.
    const size_t tbytes = (size_t)N * Cout * OH * OW * 4;
    void* tmp = nullptr;
    if (!check_cuda(cudaMallocAsync(&tmp, tbytes, ctx().stream), op, "pooled conv temporary")) return;
    int64_t tshape[4] = {N, Cout, OH, OW};
    Tensor t{};
    t.data = tmp;
    t.dtype = output->dtype;
    t.shape = tshape;
    t.ndim = 4;
    t.nbytes = (int64_t)tbytes;
    conv_impl(input, weight, bias, nullptr, &t, KH, KW, sh, sw, ph, pw, act, op);
    if (ctx().status == NNC_CUDA_OK)
      launch_maxpool_f32((const float*)tmp, (float*)output->data, N, Cout, OH, OW,
                         (int)output->shape[2], (int)output->shape[3], pool->kh, pool->kw, pool->sh,
                         pool->sw, pool->ph, pool->pw, is_nhwc(output), op);
    cudaFreeAsync(tmp, ctx().stream);
    return;
  }

  // Scratch: input planes when the input cannot be read in place (chunk
  // mode needs NHWC with C a multiple of 32; 3xTF32 needs hi/lo planes), and
  // packed weights unless prepacked.
  // (Chunk mode issues 16-byte copies: the base must be 16-byte aligned.)
  const bool in_place =
      wl.element ? !split : (is_nhwc(input) && C4 == C && !split && aligned16(input->data));
  const int64_t x_elems = wl.element ? numel(input) : (int64_t)N * H * W * C4;
  const int64_t w_elems = (int64_t)Cout * Kpad;
  size_t need = 0;
  if (!in_place) need += (size_t)(split ? 2 : 1) * ((x_elems + 63) / 64 * 64) * 4;
  if (!packed) need += (size_t)(split ? 2 : 1) * w_elems * 4;
  float* ws = nullptr;
  if (need && fixed) {
    if (need + 256 > fixed->bytes) {
      fail(NNC_CUDA_ERR_INVALID, op,
           "needs %zu bytes of scratch; the static scratch holds %zu (input %lldx%dx%dx%d, "
           "weight %dx%dx%dx%d)",
           need + 256, fixed->bytes, (long long)N, C, H, W, Cout, C, KH, KW);
      return;
    }
    ws = fixed->ptr;
  } else if (need) {
    ws = (float*)workspace(need + 256, op);
  }
  if (need && !ws) return;
  float* cur = ws;

  const float* x_hi = (const float*)input->data;
  const float* x_lo = nullptr;
  if (!in_place) {
    float* hi = cur;
    const int64_t x_span = (x_elems + 63) / 64 * 64;  // keep every plane 256-byte aligned
    float* lo = split ? cur + x_span : nullptr;
    cur += (split ? 2 : 1) * x_span;
    if (wl.element) {  // same layout, element-wise hi/lo split
      nhwc_repack_kernel<<<grid_for(x_elems, 256, 8), 256, 0, ctx().stream>>>(
          (const float*)input->data, hi, lo, x_elems, 1, 1);
    } else if (is_nhwc(input)) {
      nhwc_repack_kernel<<<grid_for(x_elems, 256, 8), 256, 0, ctx().stream>>>(
          (const float*)input->data, hi, lo, (int64_t)N * H * W, C, C4);
    } else {
      if (C4 <= 16) {
        nchw_to_nhwc_small_kernel<<<grid_for((int64_t)N * H * W, 256, 8), 256, 0, ctx().stream>>>(
            (const float*)input->data, hi, lo, N, C, (int64_t)H * W, C4);
      } else {
        const dim3 grid((unsigned)cdiv((int64_t)H * W, 32), (unsigned)cdiv(C4, 32),
                        (unsigned)(N < 65535 ? N : 65535));
        nchw_to_nhwc_pad_kernel<<<grid, 256, 0, ctx().stream>>>((const float*)input->data, hi, lo,
                                                                N, C, (int64_t)H * W, C4);
      }
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
        (const float*)weight->data, wp, Cout, C, KH, KW, C4, Kpad, split ? 1 : 0, wl.element);
    if (!check_launch(op)) return;
    w0 = wp;
    w1 = wp + w_elems;
  }

  ConvArgs g{};
  g.mode = wl.element ? kElement : kChunk;
  if (!wl.element) {
    // TMA im2col describes square windows with equal pads/strides on both
    // axes (its bounding-box corners are shared here); the corners must lie
    // in the map's signed range.
    const int lower = -ph, upper_h = (OH - 1) * sh - ph - (H - 1),
              upper_w = (OW - 1) * sw - pw - (W - 1);
    const bool square = KH == KW && sh == sw && ph == pw && upper_h == upper_w;
    if (square && lower >= -64 && upper_h >= -64 && upper_h <= 63 && sh <= 8 &&
        OH > 0 && OW > 0 && aligned16(x_hi) && (!x_lo || aligned16(x_lo)))
      g.mode = (C4 % 32 == 0) ? kIm2col128 : kIm2col16;
    if (aligned16(x_hi) && halo_eligible(C4, Cout, KH, KW, sh, sw, ph, pw, OH, OW, split))
      g.mode = kHalo;
  }
  if (is_nhwc(input)) {
    g.xs_n = (int64_t)H * W * C;
    g.xs_c = 1;
    g.xs_h = (int64_t)W * C;
    g.xs_w = C;
  } else {
    g.xs_n = (int64_t)C * H * W;
    g.xs_c = (int64_t)H * W;
    g.xs_h = W;
    g.xs_w = 1;
  }
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
  g.K = wl.K;
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

  if (g.mode == kHalo) {
    // Direct-epilogue calls take the unstaged instances, whose deeper weight
    // rings cover the weight stream's L2 latency.
    const bool direct = halo_direct(g);
    // Pair rings measured at batch 1024 (graph replay): stage-2 3 x 3 337.9
    // -> 329.7 us with 3 taps x 4 stages (against 1 x 7), stage-1 418.8 ->
    // 402.5 us with all 9 taps x 2 stages (against 3 x 5; 9 x 3 took 437.2:
    // a larger shared allocation leaves less L1).
    if (Cout > 64) {
      if (direct)
        launch_halo<128, 1, 7, 32, false, false, false, 3, 4>(g, w0, op);
      else
        launch_halo<128, 1, 4, 32>(g, w0, op);
    } else {
      if (direct)
        launch_halo<64, 3, 5, 32, false, false, false, 9, 2>(g, w0, op);
      else
        launch_halo<64, 3, 3, 32>(g, w0, op);
    }
  } else if (!split) {
    const bool pair = g.mode == kIm2col128 && conv_pair_enabled();
    // Stream-K's scratch is its own allocation: not with a fixed scratch.
    if (Cout > 128 && pair)
      launch_conv_pair<256, 6>(g, w0, op, fixed == nullptr);
    else if (Cout > 128)
      launch_conv<256, 1, 4>(g, w0, nullptr, op);
    else if (Cout > 64 && pair)
      launch_conv_pair<128, 8>(g, w0, op, fixed == nullptr);
    else if (Cout > 64)
      launch_conv<128, 1, 6>(g, w0, nullptr, op);
    else
      launch_conv<64, 1, 8>(g, w0, nullptr, op);
  } else {
    // 3xTF32: at most 128 channels per tile (two chunk buffers and the
    // running sum fit TMEM's 512 columns).
    if (Cout > 64)
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

// nnc_conv with its scratch (converted input planes, packed weights) in the
// file-scope 16 MiB g_static_scratch instead of the growable workspace:
// allocates nothing. Every byte the kernel reads from the scratch is written
// earlier in the same call, so nothing there needs clearing between calls.
void nnc_conv_static_scratch(Tensor* input, Tensor* weight, Tensor* bias, Tensor* output,
                             int kernel_h, int kernel_w, int stride_h, int stride_w, int pad_h,
                             int pad_w) {
  const char* op = "nnc_conv_static_scratch";
  OpScope s(op);
  // The device state (error word, SM count) must already exist: creating it
  // allocates, which this entry point never does.
  if (!device_ready()) {
    fail(NNC_CUDA_ERR_INVALID, op, "call nnc_cuda_init(%d) on this device first", ctx().device);
    return;
  }
  StaticScratch fixed;
  if (!static_scratch_on_device(&fixed, op)) return;
  conv_impl(input, weight, bias, nullptr, output, kernel_h, kernel_w, stride_h, stride_w, pad_h,
            pad_w, kActNone, op, &fixed);
}
void nnc_conv_relu(Tensor* input, Tensor* weight, Tensor* bias, Tensor* output, int kernel_h,
                   int kernel_w, int stride_h, int stride_w, int pad_h, int pad_w) {
  OpScope s("nnc_conv_relu");
  conv_impl(input, weight, bias, nullptr, output, kernel_h, kernel_w, stride_h, stride_w, pad_h,
            pad_w, kActRelu, "nnc_conv_relu");
}
// relu(conv) followed by max pooling in one call (no reference counterpart:
// the composition of nnc_conv_relu, ops.c:3122-3194, and nnc_maxpool2d,
// ops.c:316-391). `output` is the pooled tensor; conv_h x conv_w is the conv
// result's extent (the tensor the two reference calls would share).
void nnc_conv_relu_maxpool(Tensor* input, Tensor* weight, Tensor* bias, Tensor* output,
                           int kernel_h, int kernel_w, int stride_h, int stride_w, int pad_h,
                           int pad_w, int conv_h, int conv_w, int pool_kh, int pool_kw,
                           int pool_sh, int pool_sw, int pool_ph, int pool_pw) {
  const char* op = "nnc_conv_relu_maxpool";
  OpScope s(op);
  const PoolSpec pool{conv_h, conv_w, pool_kh, pool_kw, pool_sh, pool_sw, pool_ph, pool_pw};
  conv_impl(input, weight, bias, nullptr, output, kernel_h, kernel_w, stride_h, stride_w, pad_h,
            pad_w, kActRelu, op, nullptr, &pool);
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
  const WeightLayout wl = weight_layout((int)w->shape[1], (int)w->shape[2], (int)w->shape[3]);
  return (size_t)2 * w->shape[0] * wl.Kpad * 4;
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
  const WeightLayout wl = weight_layout(Cin, KH, KW);
  const int64_t total = (int64_t)Cout * wl.Kpad;
  pack_weight_kernel<<<grid_for(total, 256, 8), 256, 0, ctx().stream>>>(
      (const float*)w->data, (float*)dst, Cout, Cin, KH, KW, wl.C4, wl.Kpad, 1, wl.element);
  if (!check_launch(op)) return ctx().status;
  w->data = dst;
  w->dtype = (nnc_dtype_t)((int)w->dtype | NNC_CUDA_TAG_PACKED_CONV);
  return NNC_CUDA_OK;
}

}  // extern "C"
