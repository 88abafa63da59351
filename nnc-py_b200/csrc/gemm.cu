// Dense contractions: nnc_gemm / nnc_gemm_nt / nnc_matmul (+ relu variants)
// on the sm_100a tensor cores (tcgen05.mma kind::tf32, accumulators in TMEM,
// operands staged by TMA).
//
// Kernel shape (persistent, one CTA per SM, 192 threads):
//   warp 0      TMA producer: streams 128 x 32 A tiles and BN x 32 B tiles
//               (both K-major, 128-byte swizzle) into a STAGES-deep ring;
//   warp 1      allocates TMEM and issues the MMAs (one thread), 4 k-steps of
//               K = 8 per 32-wide stage; commits free the ring slots;
//   warps 2..5  epilogue: tcgen05.ld of the 128 x BN fp32 accumulator,
//               alpha / beta*C / relu, stores to global.
// Two TMEM accumulators (2 x BN columns) let tile i's epilogue overlap tile
// i+1's main loop.
//
// Precision: TF32 mode issues one MMA per k-step. 3xTF32 mode splits A and B
// into hi = tf32(x) and lo = x - hi planes and issues lo*hi + hi*lo + hi*hi,
// which recovers ~fp32 accuracy (the reference accumulates in fp64,
// ops.c:1800-1840). Shapes the TMA path cannot take (K % 4 != 0, unaligned
// bases, very small M or N) go to a SIMT kernel with fp64 accumulation.
#include <math.h>
#include <stdlib.h>

#include "common.cuh"
#include "movement.cuh"
#include "tc.cuh"

namespace nnc {
namespace {

constexpr int BM = 128;
constexpr int BK = 32;  // fp32 elements per 128-byte swizzle row
constexpr int kTCThreads = 192;

struct GemmArgs {
  int M, N, K;
  int m_tiles, n_tiles;
  int64_t tiles;
  int a_batched, b_batched;
  float alpha, beta;
  const float* C;
  int c_mode;  // 0: none, 1: C[n] (1-D), 2: C[m * ldc + n]
  int64_t ldc, c_batch_stride;
  float* D;
  int64_t ldd, d_batch_stride;
  int relu;
  int tma_store;  // 1: D written by TMA stores through tmD (dense, 16-byte rows)
  int b_mn;       // 1: B tiles are MN-major ({32 n, 32 k} boxes of a [K, N] matrix)
  int pair_b;     // CTA pairs only: 1 = the two CTAs take consecutive batches (M <= 128)
  int softmax;    // 1: each output row is replaced by the softmax of alpha * row (N <= BN)
  int batches;
  int* err;
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return (uint8_t*)(((uintptr_t)p + 1023) & ~(uintptr_t)1023);
}

template <int BN, int SPLIT, int STAGES>
struct GemmCfg {
  static constexpr uint32_t A_BYTES = BM * BK * 4;
  static constexpr uint32_t B_BYTES = BN * BK * 4;
  static constexpr uint32_t STAGE_BYTES = SPLIT * (A_BYTES + B_BYTES);
  // Two accumulators (a power of two for BN in {64, 128, 256}); in 3xTF32
  // mode two chunk buffers plus the running sum (tc::promote_chunk32),
  // rounded up to a power of two.
  static constexpr uint32_t TMEM_COLS = SPLIT == 1 ? 2 * BN : (3 * BN <= 256 ? 256 : 512);
  // Epilogue staging: per epilogue warp two 32 x 32 fp32 boxes (4 KB each).
  static constexpr uint32_t STAGING_BYTES = 4 * 2 * 4096;
  static constexpr size_t SMEM =
      (size_t)STAGES * STAGE_BYTES + STAGING_BYTES + 1024 /*align*/ + 256 /*bars*/;
};

// Epilogue of one accumulator tile for one warp: TMEM lanes [32 quad, +32)
// hold rows row0 .. row0 + 31 of batch b; columns nt * BN + [0, BN) in
// 32-column slices: alpha, beta * C, relu, then a TMA store of a 32 x 32
// shared box (tma_store; two boxes at box0, alternated through bsel) or
// per-thread row stores.
template <int BN>
__device__ __forceinline__ void store_slices(const GemmArgs& g, const CUtensorMap* tmD,
                                             uint32_t tmem_base, int acc, int quad, int lane,
                                             int row0, int nt, int b, float* box0, int& bsel,
                                             bool vec_ok, float alpha) {
  const int row = row0 + lane;
  float* drow = g.D + (int64_t)b * g.d_batch_stride + (int64_t)row * g.ldd;
  const float* crow = nullptr;
  if (g.c_mode == 2) crow = g.C + (int64_t)b * g.c_batch_stride + (int64_t)row * g.ldc;
#pragma unroll 1
  for (int c0 = 0; c0 < BN; c0 += 32) {
    const int n0 = nt * BN + c0;
    if (n0 >= g.N) break;  // warp-uniform
    uint32_t r[32];
    __syncwarp();  // tcgen05.ld is .sync.aligned: the warp must be converged
    const uint32_t taddr = tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BN + c0;
    tc::tmem_ld16(taddr, *reinterpret_cast<uint32_t(*)[16]>(&r[0]));
    tc::tmem_ld16(taddr + 16, *reinterpret_cast<uint32_t(*)[16]>(&r[16]));
    tc::tmem_ld_wait();
    // The modes are tested once per slice, outside the element loops: a
    // per-element test of c_mode with its guarded loads cost ~2,900
    // cycles per 32-column slice (measured), 30x the TMEM load.
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = alpha * __uint_as_float(r[j]);
    if (g.c_mode == 1) {  // C[n], the same 32 values for every lane (broadcast loads)
      const float* cb = g.C + n0;
      if (n0 + 32 <= g.N && ((uintptr_t)cb & 15) == 0) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 c4 = __ldg(reinterpret_cast<const float4*>(cb) + j);
          v[4 * j] = fmaf(g.beta, c4.x, v[4 * j]);
          v[4 * j + 1] = fmaf(g.beta, c4.y, v[4 * j + 1]);
          v[4 * j + 2] = fmaf(g.beta, c4.z, v[4 * j + 2]);
          v[4 * j + 3] = fmaf(g.beta, c4.w, v[4 * j + 3]);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (n0 + j < g.N) v[j] = fmaf(g.beta, __ldg(cb + j), v[j]);
      }
    } else if (g.c_mode == 2 && row < g.M) {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (n0 + j < g.N) v[j] = fmaf(g.beta, crow[n0 + j], v[j]);
    }
    if (g.relu) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = v[j] > 0.0f ? v[j] : 0.0f;
    }
    if (g.tma_store) {
      if (row0 >= g.M) continue;  // warp-uniform: the whole box lies below M
      float* box = box0 + bsel * 1024;
      if (lane == 0) tc::bulk_wait_group_read<1>();  // the store 2 slices ago read `box`
      __syncwarp();
      float4* brow = reinterpret_cast<float4*>(box + lane * 32);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        brow[j ^ (lane & 7)] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
      tc::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tc::tma_store_3d(tmD, box, n0, row0, b);
        tc::bulk_commit_group();
      }
      bsel ^= 1;
    } else if (row < g.M) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int nh = n0 + 16 * h;
        if (vec_ok && nh + 16 <= g.N) {
          float4* d4 = reinterpret_cast<float4*>(drow + nh);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            d4[j] = make_float4(v[16 * h + 4 * j], v[16 * h + 4 * j + 1],
                                v[16 * h + 4 * j + 2], v[16 * h + 4 * j + 3]);
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (nh + j < g.N) drow[nh + j] = v[16 * h + j];
        }
      }
    }
  }
}

// Row softmax in the epilogue (nnc_matmul_scale_softmax): this warp's 32
// TMEM lanes hold 32 output rows whose N <= BN columns are all in this tile.
// Each thread takes its row through three passes over the accumulator, in
// column order as the reference's nnc_softmax does (ops.c:283-307): the max
// of v = alpha * acc; e = expf(v - max) with a sequential fp32 sum, e
// written back over the accumulator; then e / sum written back, which the
// ordinary epilogue stores with alpha 1.
template <int BN>
__device__ __forceinline__ void softmax_rows_tmem(uint32_t lane_addr, uint32_t col0, int N,
                                                  float alpha) {
  float mx = -INFINITY;
#pragma unroll 1
  for (int c0 = 0; c0 < BN && c0 < N; c0 += 16) {
    uint32_t r[16];
    tc::tmem_ld16(lane_addr + col0 + c0, r);
    tc::tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float v = alpha * __uint_as_float(r[j]);
      if (c0 + j < N && v > mx) mx = v;
    }
  }
  float sum = 0.0f;
#pragma unroll 1
  for (int c0 = 0; c0 < BN && c0 < N; c0 += 16) {
    uint32_t r[16];
    tc::tmem_ld16(lane_addr + col0 + c0, r);
    tc::tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float e = expf(alpha * __uint_as_float(r[j]) - mx);
      if (c0 + j < N) sum = __fadd_rn(sum, e);
      r[j] = __float_as_uint(e);
    }
    tc::tmem_st16(lane_addr + col0 + c0, r);
  }
  tc::tmem_st_wait();
#pragma unroll 1
  for (int c0 = 0; c0 < BN && c0 < N; c0 += 16) {
    uint32_t r[16];
    tc::tmem_ld16(lane_addr + col0 + c0, r);
    tc::tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 16; ++j) r[j] = __float_as_uint(__fdiv_rn(__uint_as_float(r[j]), sum));
    tc::tmem_st16(lane_addr + col0 + c0, r);
  }
  tc::tmem_st_wait();
}

template <int BN, int SPLIT, int STAGES>
__global__ void __launch_bounds__(kTCThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA0, const __grid_constant__ CUtensorMap tmA1,
                   const __grid_constant__ CUtensorMap tmB0, const __grid_constant__ CUtensorMap tmB1,
                   const __grid_constant__ CUtensorMap tmD, const GemmArgs g) {
  using Cfg = GemmCfg<BN, SPLIT, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  pdl_trigger();
  uint8_t* smem = align1024(smem_raw);
  float* staging = reinterpret_cast<float*>(smem + STAGES * Cfg::STAGE_BYTES);
  uint64_t* full =
      reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES + Cfg::STAGING_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* done = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kblocks = (g.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      tc::mbar_init(&tfull[a], 1);
      tc::mbar_init(&tempty[a], 4);
    }
    tc::mbar_init(done, 1);
    tc::fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tc::prefetch_tmap(&tmA0);
    tc::prefetch_tmap(&tmB0);
    if (SPLIT == 2) {
      tc::prefetch_tmap(&tmA1);
      tc::prefetch_tmap(&tmB1);
    }
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // the previous kernel's outputs are complete from here on

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; t < g.tiles && ok; t += gridDim.x) {
        const int per_b = g.m_tiles * g.n_tiles;
        const int b = (int)(t / per_b);
        const int mt = (int)((t % per_b) / g.n_tiles), nt = (int)((t % per_b) % g.n_tiles);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!tc::mbar_wait(&empty[stage], phase ^ 1, g.err)) {
            ok = false;
            break;
          }
          uint8_t* s = smem + stage * Cfg::STAGE_BYTES;
          tc::mbar_arrive_expect_tx(&full[stage], Cfg::STAGE_BYTES);
          const int kx = kb * BK;
          tc::tma_load_3d(s, &tmA0, &full[stage], kx, mt * BM, b * g.a_batched);
          if (SPLIT == 2)
            tc::tma_load_3d(s + Cfg::A_BYTES, &tmA1, &full[stage], kx, mt * BM, b * g.a_batched);
          uint8_t* sb = s + SPLIT * Cfg::A_BYTES;
          if (g.b_mn) {
#pragma unroll
            for (int c = 0; c < BN / 32; ++c) {
              tc::tma_load_3d(sb + c * 4096, &tmB0, &full[stage], nt * BN + 32 * c, kx,
                              b * g.b_batched);
              if (SPLIT == 2)
                tc::tma_load_3d(sb + Cfg::B_BYTES + c * 4096, &tmB1, &full[stage],
                                nt * BN + 32 * c, kx, b * g.b_batched);
            }
          } else {
            tc::tma_load_3d(sb, &tmB0, &full[stage], kx, nt * BN, b * g.b_batched);
            if (SPLIT == 2)
              tc::tma_load_3d(sb + Cfg::B_BYTES, &tmB1, &full[stage], kx, nt * BN,
                              b * g.b_batched);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      const uint32_t idesc = tc::idesc_tf32(BM, BN) | (g.b_mn ? tc::kIdescBMajorMN : 0u);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;  // accumulator fills so far (tiles, or 3xTF32 chunks)
      bool ok = true;
      // 3xTF32: each chunk of kChunkKBlocks k-blocks starts a fresh
      // accumulator in the next buffer (see tc::promote_chunk32).
      const int chunk_kb = SPLIT == 2 ? tc::kChunkKBlocks : kblocks;
      const int chunks = SPLIT == 2 ? (kblocks + chunk_kb - 1) / chunk_kb : 1;
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
        const int kend = kc + chunk_kb < kblocks ? kc + chunk_kb : kblocks;
        for (int kb = kc; kb < kend; ++kb) {
          if (!tc::mbar_wait(&full[stage], phase, g.err)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t sa = tc::smem_u32(smem + stage * Cfg::STAGE_BYTES);
          const uint32_t sb = sa + SPLIT * Cfg::A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 8; ++k) {
            const uint64_t a0 = tc::desc_kmajor_sw128(sa + k * 32);
            const uint64_t b0 = g.b_mn ? tc::desc_mn_sw128_atom32(sb + k * 1024, 4096)
                                       : tc::desc_kmajor_sw128(sb + k * 32);
            const uint32_t first = ((kb - kc) | k) != 0;
            if (SPLIT == 1) {
              tc::mma_tf32(d_tmem, a0, b0, idesc, first);
            } else {
              const uint64_t a1 = tc::desc_kmajor_sw128(sa + Cfg::A_BYTES + k * 32);
              const uint64_t b1 = g.b_mn ? tc::desc_mn_sw128_atom32(sb + Cfg::B_BYTES + k * 1024, 4096)
                                         : tc::desc_kmajor_sw128(sb + Cfg::B_BYTES + k * 32);
              tc::mma_tf32(d_tmem, a1, b0, idesc, first);  // lo * hi
              tc::mma_tf32(d_tmem, a0, b1, idesc, 1);      // hi * lo
              tc::mma_tf32(d_tmem, a0, b0, idesc, 1);      // hi * hi
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
      // Drain: every MMA issued above has completed once `done` fires.
      tc::mma_commit(done);
      tc::mbar_wait(done, 0, g.err);
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    // Each warp owns TMEM lanes (rows) [32*quad, 32*quad + 32). With tma_store
    // it writes 32-column slices of its rows into a 128-byte-swizzled 32 x 32
    // shared box (conflict-free: lane r puts 16-byte chunk j at j ^ (r & 7))
    // and one lane stores the box with TMA, double-buffered; otherwise each
    // thread stores its own row.
    const int quad = warp & 3;  // TMEM lanes [32*quad, 32*quad + 32)
    int local = 0;
    const bool vec_ok = ((g.ldd & 3) == 0) && ((((uintptr_t)g.D) & 15) == 0);
    float* box0 = staging + quad * 2 * 1024;
    int bsel = 0;
    if constexpr (SPLIT == 1) {
      for (int64_t t = blockIdx.x; t < g.tiles; t += gridDim.x, ++local) {
        const int per_b = g.m_tiles * g.n_tiles;
        const int b = (int)(t / per_b);
        const int mt = (int)((t % per_b) / g.n_tiles), nt = (int)((t % per_b) % g.n_tiles);
        const int acc = local & 1;
        const uint32_t aphase = (local >> 1) & 1;
        if (!tc::mbar_wait(&tfull[acc], aphase, g.err)) break;
        tc::tc_fence_after();
        float alpha = g.alpha;
        if (g.softmax) {
          softmax_rows_tmem<BN>(tmem_base + ((uint32_t)(quad * 32) << 16), acc * BN, g.N, g.alpha);
          alpha = 1.0f;
        }
        store_slices<BN>(g, &tmD, tmem_base, acc, quad, lane, mt * BM + quad * 32, nt, b, box0,
                         bsel, vec_ok, alpha);
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&tempty[acc]);
      }
    } else {
      // 3xTF32: every chunk's partial sums are folded into the running sum
      // (columns 2 BN + c); the last chunk's buffer receives the total and
      // is stored as usual.
      const uint32_t lane_addr = tmem_base + ((uint32_t)(quad * 32) << 16);
      bool ok = true;
      for (int64_t t = blockIdx.x; t < g.tiles && ok; t += gridDim.x) {
        const int per_b = g.m_tiles * g.n_tiles;
        const int b = (int)(t / per_b);
        const int mt = (int)((t % per_b) / g.n_tiles), nt = (int)((t % per_b) % g.n_tiles);
        for (int kc = 0; kc < kblocks; kc += tc::kChunkKBlocks, ++local) {
          const int acc = local & 1;
          const uint32_t aphase = (local >> 1) & 1;
          if (!tc::mbar_wait(&tfull[acc], aphase, g.err)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const bool last = kc + tc::kChunkKBlocks >= kblocks;
          if (!(kc == 0 && last)) {
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 32) {
              if (nt * BN + c0 >= g.N) break;  // warp-uniform
              tc::promote_chunk32(lane_addr, acc * BN + c0, 2 * BN + c0, kc == 0, last);
            }
            tc::tmem_st_wait();
          }
          if (last) {
            float alpha = g.alpha;
            if (g.softmax) {
              softmax_rows_tmem<BN>(lane_addr, acc * BN, g.N, g.alpha);
              alpha = 1.0f;
            }
            store_slices<BN>(g, &tmD, tmem_base, acc, quad, lane, mt * BM + quad * 32, nt, b, box0,
                             bsel, vec_ok, alpha);
          }
          tc::tc_fence_before();
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(&tempty[acc]);
        }
      }
    }
    if (g.tma_store && lane == 0) tc::bulk_wait_group<0>();
  }

  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// ------------------------------------------------------- CTA pairs ----
//
// TF32 problems with N > 128 and enough 256-row tiles to occupy the SMs run on
// CTA pairs (tcgen05 cta_group::2): a cluster of two CTAs computes a 256 x BN
// tile. CTA r loads rows [m0 + 128 r, +128) of A and its half of the tile's
// B (BN / 2 rows of a [N, K] B, or BN / 2 columns of a [K, N] B); the even
// CTA issues M = 256 MMAs that read both CTAs' operands at the same shared
// offsets, each CTA's TMEM holding its 128 rows x BN columns. Per k-block an
// SM receives 16 + 16 KB for 512 MMA cycles (the single-CTA kernel's BN = 256
// tiles need 16 + 32 KB, more than the ~80 B/clk TMA delivers per SM).
// Barriers as in the conv pair kernel: the even CTA's full[s] counts both
// CTAs' bytes, its commits arrive in both CTAs (empty, tfull, done), and all
// eight epilogue warps arrive on the even CTA's tempty. Rows past M are zero
// filled by TMA and clipped by the TMA stores. No load uses cluster multicast.
template <int BN, int STAGES>
struct GemmPairCfg {
  static constexpr uint32_t A_BYTES = BM * BK * 4;         // 16 KB
  static constexpr uint32_t B_BYTES = (BN / 2) * BK * 4;   // this CTA's half of B
  static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr uint32_t TMEM_COLS = 2 * BN;
  static constexpr uint32_t STAGING_BYTES = 4 * 2 * 4096;
  static constexpr size_t SMEM =
      (size_t)STAGES * STAGE_BYTES + STAGING_BYTES + 1024 /*align*/ + 256 /*bars*/;
};

template <int BN, int STAGES>
__global__ void __launch_bounds__(kTCThreads, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmD, const GemmArgs g) {
  using Cfg = GemmPairCfg<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  pdl_trigger();
  uint8_t* smem = align1024(smem_raw);
  float* staging = reinterpret_cast<float*>(smem + STAGES * Cfg::STAGE_BYTES);
  uint64_t* full =
      reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES + Cfg::STAGING_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* done = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = tc::cluster_ctarank();  // 0: issues the MMAs
  const int64_t cluster = blockIdx.x >> 1, clusters = gridDim.x >> 1;
  const int kblocks = (g.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      tc::mbar_init(&tfull[a], 1);
      tc::mbar_init(&tempty[a], 8);  // even CTA: both CTAs' four epilogue warps
    }
    tc::mbar_init(done, 1);
    tc::fence_barrier_init();
    tc::prefetch_tmap(&tmA);
    tc::prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    tc::tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
    tc::tmem_relinquish_pair();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::cluster_sync();  // both CTAs' barriers initialised, TMEM allocated
  tc::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // the previous kernel's outputs are complete from here on
  const int per_b = g.m_tiles * g.n_tiles;  // m_tiles counts 256-row tiles here

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer (one thread per CTA) ----------------
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int64_t t = cluster; t < g.tiles && ok; t += clusters) {
        // Pair tile: 256 rows of one batch, or (pair_b) rows 0..127 of
        // batches 2 j and 2 j + 1, one per CTA (a batch past the last is
        // read as zeros and not stored).
        const int b = g.pair_b ? (int)(t / g.n_tiles) * 2 + (int)rank : (int)(t / per_b);
        const int mt = g.pair_b ? 0 : (int)((t % per_b) / g.n_tiles);
        const int nt = (int)((g.pair_b ? t : t % per_b) % g.n_tiles);
        const int row0 = g.pair_b ? 0 : mt * (2 * BM) + (int)rank * BM;
        const int n_half = nt * BN + (int)rank * (BN / 2);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!tc::mbar_wait(&empty[stage], phase ^ 1, g.err)) {
            ok = false;
            break;
          }
          uint8_t* s = smem + stage * Cfg::STAGE_BYTES;
          if (rank == 0) tc::mbar_arrive_expect_tx(&full[stage], 2 * Cfg::STAGE_BYTES);
          const uint32_t bar = tc::mapa(tc::smem_u32(&full[stage]), 0);
          const int kx = kb * BK;
          tc::tma_load_3d_pair(s, &tmA, bar, kx, row0, b * g.a_batched);
          uint8_t* sb = s + Cfg::A_BYTES;
          if (g.b_mn) {
#pragma unroll
            for (int c = 0; c < BN / 64; ++c)
              tc::tma_load_3d_pair(sb + c * 4096, &tmB, bar, n_half + 32 * c, kx, b * g.b_batched);
          } else {
            tc::tma_load_3d_pair(sb, &tmB, bar, kx, n_half, b * g.b_batched);
          }
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
  } else if (warp == 1) {
    if (rank == 0 && lane == 0) {
      // ---------------- MMA issuer (even CTA) ----------------
      const uint32_t idesc = tc::idesc_tf32(2 * BM, BN) | (g.b_mn ? tc::kIdescBMajorMN : 0u);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int64_t t = cluster; t < g.tiles && ok; t += clusters, ++local) {
        const int acc = local & 1;
        const uint32_t aphase = (local >> 1) & 1;
        if (!tc::mbar_wait(&tempty[acc], aphase ^ 1, g.err)) break;
        tc::tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!tc::mbar_wait(&full[stage], phase, g.err)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t sa = tc::smem_u32(smem + stage * Cfg::STAGE_BYTES);
          const uint32_t sb = sa + Cfg::A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 8; ++k) {
            const uint64_t bd = g.b_mn ? tc::desc_mn_sw128_atom32(sb + k * 1024, 4096)
                                       : tc::desc_kmajor_sw128(sb + k * 32);
            tc::mma_tf32_pair(d_tmem, tc::desc_kmajor_sw128(sa + k * 32), bd, idesc,
                              (kb | k) != 0);
          }
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
    // ---------------- epilogue (warps 2..5 of both CTAs) ----------------
    const int quad = warp & 3;
    float* box0 = staging + quad * 2 * 1024;
    int bsel = 0;
    const uint32_t tempty0 = tc::mapa(tc::smem_u32(&tempty[0]), 0);
    int local = 0;
    for (int64_t t = cluster; t < g.tiles; t += clusters, ++local) {
      const int b = g.pair_b ? (int)(t / g.n_tiles) * 2 + (int)rank : (int)(t / per_b);
      const int mt = g.pair_b ? 0 : (int)((t % per_b) / g.n_tiles);
      const int nt = (int)((g.pair_b ? t : t % per_b) % g.n_tiles);
      const int acc = local & 1;
      const uint32_t aphase = (local >> 1) & 1;
      if (!tc::mbar_wait(&tfull[acc], aphase, g.err)) break;
      tc::tc_fence_after();
      const int row0 = g.pair_b ? quad * 32 : mt * (2 * BM) + (int)rank * BM + quad * 32;
      // (a missing last batch still takes part: its TMEM loads are warp-wide)
      store_slices<BN>(g, &tmD, tmem_base, acc, quad, lane, b < g.batches ? row0 : g.M, nt, b, box0,
                       bsel, true, g.alpha);
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive_cluster(tempty0 + acc * (uint32_t)sizeof(uint64_t));
    }
    if (lane == 0) tc::bulk_wait_group<0>();
    // The odd CTA leaves only after the even CTA's last commit has arrived
    // here (its barriers receive the pair's commits).
    if (rank == 1 && warp == 2) tc::mbar_wait_warp(done, 0, g.err);
  }

  tc::tc_fence_before();
  __syncthreads();
  tc::cluster_sync();  // no CTA frees the pair's TMEM or leaves while the other works
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
  }
}

// hi = tf32(x), lo = x - hi (exact in fp32), for matrices of `mat` elements
// read at x + b * in_bs and written densely.
__global__ void __launch_bounds__(256) split_tf32_kernel(const float* __restrict__ x,
                                                         int64_t in_bs, float* __restrict__ hi,
                                                         float* __restrict__ lo, int64_t mat,
                                                         int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float v = x[(i / mat) * in_bs + i % mat];
    const float h = tc::to_tf32(v);
    hi[i] = h;
    lo[i] = v - h;
  }
}

// SIMT fallback: one output per thread, fp64 accumulation over K with
// generic strides (covers every transpose mode, vectors, odd K).
struct SimtArgs {
  int M, N, K, batches;
  const float* A;
  int64_t sam, sak, a_bs;
  const float* B;
  int64_t sbk, sbn, b_bs;
  float alpha, beta;
  const float* C;
  int c_mode;
  int64_t ldc, c_bs;
  float* D;
  int64_t ldd, d_bs;
  int relu;
};

__global__ void __launch_bounds__(256) gemm_simt_kernel(const SimtArgs a) {
  constexpr int T = 16;
  __shared__ float As[T][T + 1];
  __shared__ float Bs[T][T + 1];
  const int tx = threadIdx.x % T, ty = threadIdx.x / T;
  const int64_t tiles_m = cdiv(a.M, T), tiles_n = cdiv(a.N, T);
  for (int64_t t = blockIdx.x; t < (int64_t)a.batches * tiles_m * tiles_n; t += gridDim.x) {
    const int64_t b = t / (tiles_m * tiles_n);
    const int64_t rem = t % (tiles_m * tiles_n);
    const int m = (int)(rem / tiles_n) * T + ty, n = (int)(rem % tiles_n) * T + tx;
    const float* A = a.A + b * a.a_bs;
    const float* B = a.B + b * a.b_bs;
    double acc = 0.0;
    for (int k0 = 0; k0 < a.K; k0 += T) {
      const int am = (int)(rem / tiles_n) * T + ty, ak = k0 + tx;
      As[ty][tx] = (am < a.M && ak < a.K) ? A[am * a.sam + ak * a.sak] : 0.0f;
      const int bk = k0 + ty, bn = (int)(rem % tiles_n) * T + tx;
      Bs[ty][tx] = (bk < a.K && bn < a.N) ? B[bk * a.sbk + bn * a.sbn] : 0.0f;
      __syncthreads();
#pragma unroll
      for (int k = 0; k < T; ++k) acc += (double)As[ty][k] * (double)Bs[k][tx];
      __syncthreads();
    }
    if (m < a.M && n < a.N) {
      acc *= (double)a.alpha;
      if (a.c_mode == 1) acc += (double)a.beta * (double)a.C[n];
      if (a.c_mode == 2) acc += (double)a.beta * (double)a.C[b * a.c_bs + (int64_t)m * a.ldc + n];
      float o = (float)acc;
      if (a.relu) o = o > 0.0f ? o : 0.0f;
      a.D[b * a.d_bs + (int64_t)m * a.ldd + n] = o;
    }
  }
}

// ------------------------------------------------------------------ host --

// A contraction after shape analysis: D[b] = alpha * op(A[b]) op(B[b]) + beta * C.
struct Problem {
  int M, N, K, batches;
  const float* A;
  bool a_trans;  // A stored [K, M] instead of [M, K]
  int64_t a_bs;  // batch stride in elements (0 = broadcast)
  const float* B;
  bool b_kmajor;  // B stored [N, K] (K-major) instead of [K, N]
  int64_t b_bs;
  float alpha, beta;
  const float* C;
  int c_mode;
  int64_t ldc, c_bs;
  float* D;
  int64_t d_bs;
  int relu;
  int softmax;  // row softmax of alpha * A B in the epilogue (N <= 128, see run_problem)
};

template <int BN, int SPLIT, int STAGES>
bool launch_tc(const Problem& p, const float* A0, const float* A1, const float* B0,
               const float* B1, const char* op) {
  using Cfg = GemmCfg<BN, SPLIT, STAGES>;
  CUtensorMap ta0, ta1, tb0, tb1;
  const uint64_t a_dims[3] = {(uint64_t)p.K, (uint64_t)p.M, (uint64_t)(p.a_bs ? p.batches : 1)};
  const uint64_t a_str[2] = {(uint64_t)p.K * 4, (uint64_t)(p.a_bs ? p.a_bs : (int64_t)p.M * p.K) * 4};
  // B: K-major [N, K] rows, or MN-major [K, N] rows read as {32 n, BK k} boxes.
  const bool mn = !p.b_kmajor;
  const uint64_t b_dims[3] = {(uint64_t)(mn ? p.N : p.K), (uint64_t)(mn ? p.K : p.N),
                              (uint64_t)(p.b_bs ? p.batches : 1)};
  const uint64_t b_str[2] = {(uint64_t)(mn ? p.N : p.K) * 4,
                             (uint64_t)(p.b_bs ? p.b_bs : (int64_t)p.N * p.K) * 4};
  const uint32_t a_box[3] = {BK, BM, 1};
  const uint32_t b_box[3] = {mn ? 32u : (uint32_t)BK, mn ? (uint32_t)BK : (uint32_t)BN, 1};
  if (!encode_tmap_f32(&ta0, A0, 3, a_dims, a_str, a_box, nullptr, op)) return false;
  const int b_swz = mn ? kSwizzle128Atom32 : 128;
  if (!encode_tmap_f32(&tb0, B0, 3, b_dims, b_str, b_box, nullptr, op, b_swz)) return false;
  ta1 = ta0;
  tb1 = tb0;
  if (SPLIT == 2) {
    if (!encode_tmap_f32(&ta1, A1, 3, a_dims, a_str, a_box, nullptr, op)) return false;
    if (!encode_tmap_f32(&tb1, B1, 3, b_dims, b_str, b_box, nullptr, op, b_swz)) return false;
  }
  // D through TMA stores when its rows and batches start on 16-byte
  // boundaries (N % 4 == 0, aligned base); 32 x 32 boxes, 128-byte swizzle.
  CUtensorMap td = ta0;
  const bool tma_store = (p.N % 4 == 0) && (p.d_bs % 4 == 0) && aligned16(p.D);
  if (tma_store) {
    const uint64_t d_dims[3] = {(uint64_t)p.N, (uint64_t)p.M, (uint64_t)p.batches};
    const uint64_t d_str[2] = {(uint64_t)p.N * 4,
                               (uint64_t)(p.batches > 1 ? p.d_bs : (int64_t)p.M * p.N) * 4};
    const uint32_t d_box[3] = {32, 32, 1};
    if (!encode_tmap_f32(&td, p.D, 3, d_dims, d_str, d_box, nullptr, op)) return false;
  }
  GemmArgs g;
  g.M = p.M;
  g.N = p.N;
  g.K = p.K;
  g.m_tiles = (int)cdiv(p.M, BM);
  g.n_tiles = (int)cdiv(p.N, BN);
  g.tiles = (int64_t)p.batches * g.m_tiles * g.n_tiles;
  g.a_batched = p.a_bs ? 1 : 0;
  g.b_batched = p.b_bs ? 1 : 0;
  g.alpha = p.alpha;
  g.beta = p.beta;
  g.C = p.C;
  g.c_mode = p.c_mode;
  g.ldc = p.ldc;
  g.c_batch_stride = p.c_bs;
  g.D = p.D;
  g.ldd = p.N;
  g.d_batch_stride = p.d_bs;
  g.relu = p.relu;
  g.pair_b = 0;
  g.softmax = p.softmax;
  g.batches = p.batches;
  g.tma_store = tma_store ? 1 : 0;
  g.b_mn = mn ? 1 : 0;
  g.err = device_error_word();
  auto kern = gemm_tc_kernel<BN, SPLIT, STAGES>;
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
  launch_pdl(kern, grid, kTCThreads, Cfg::SMEM, ta0, ta1, tb0, tb1, td, g);
  return check_launch(op);
}

// CTA-pair launch (TF32, D written by TMA stores): see gemm_tc2_kernel.
template <int BN, int STAGES>
bool launch_tc2(const Problem& p, const float* A, const float* B, const char* op,
                bool pair_batches = false) {
  using Cfg = GemmPairCfg<BN, STAGES>;
  CUtensorMap ta, tb, td;
  const uint64_t a_dims[3] = {(uint64_t)p.K, (uint64_t)p.M, (uint64_t)(p.a_bs ? p.batches : 1)};
  const uint64_t a_str[2] = {(uint64_t)p.K * 4, (uint64_t)(p.a_bs ? p.a_bs : (int64_t)p.M * p.K) * 4};
  const uint32_t a_box[3] = {BK, BM, 1};
  if (!encode_tmap_f32(&ta, A, 3, a_dims, a_str, a_box, nullptr, op)) return false;
  const bool mn = !p.b_kmajor;
  const uint64_t b_dims[3] = {(uint64_t)(mn ? p.N : p.K), (uint64_t)(mn ? p.K : p.N),
                              (uint64_t)(p.b_bs ? p.batches : 1)};
  const uint64_t b_str[2] = {(uint64_t)(mn ? p.N : p.K) * 4,
                             (uint64_t)(p.b_bs ? p.b_bs : (int64_t)p.N * p.K) * 4};
  const uint32_t b_box[3] = {mn ? 32u : (uint32_t)BK, mn ? (uint32_t)BK : (uint32_t)(BN / 2), 1};
  if (!encode_tmap_f32(&tb, B, 3, b_dims, b_str, b_box, nullptr, op, mn ? kSwizzle128Atom32 : 128))
    return false;
  const uint64_t d_dims[3] = {(uint64_t)p.N, (uint64_t)p.M, (uint64_t)p.batches};
  const uint64_t d_str[2] = {(uint64_t)p.N * 4,
                             (uint64_t)(p.batches > 1 ? p.d_bs : (int64_t)p.M * p.N) * 4};
  const uint32_t d_box[3] = {32, 32, 1};
  if (!encode_tmap_f32(&td, p.D, 3, d_dims, d_str, d_box, nullptr, op)) return false;
  GemmArgs g;
  g.M = p.M;
  g.N = p.N;
  g.K = p.K;
  g.pair_b = pair_batches ? 1 : 0;
  g.softmax = 0;
  g.batches = p.batches;
  g.m_tiles = pair_batches ? 1 : (int)cdiv(p.M, 2 * BM);
  g.n_tiles = (int)cdiv(p.N, BN);
  g.tiles = (pair_batches ? (int64_t)(p.batches + 1) / 2 : (int64_t)p.batches * g.m_tiles) * g.n_tiles;
  g.a_batched = p.a_bs ? 1 : 0;
  g.b_batched = p.b_bs ? 1 : 0;
  g.alpha = p.alpha;
  g.beta = p.beta;
  g.C = p.C;
  g.c_mode = p.c_mode;
  g.ldc = p.ldc;
  g.c_batch_stride = p.c_bs;
  g.D = p.D;
  g.ldd = p.N;
  g.d_batch_stride = p.d_bs;
  g.relu = p.relu;
  g.tma_store = 1;
  g.b_mn = mn ? 1 : 0;
  g.err = device_error_word();
  auto kern = gemm_tc2_kernel<BN, STAGES>;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kTCThreads, 1, 1);
  cfg.dynamicSmemBytes = Cfg::SMEM;
  cfg.stream = ctx().stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  static bool attr_set[64] = {};
  static int max_pairs[64] = {};
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
    max_pairs[ctx().device] = n;
    attr_set[ctx().device] = true;
  }
  const int64_t pairs = g.tiles < max_pairs[ctx().device] ? g.tiles : max_pairs[ctx().device];
  cfg.gridDim = dim3((unsigned)(2 * pairs), 1, 1);
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see pdl_trigger
  attr[1].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.numAttrs = 2;
  if (!check_cuda(cudaLaunchKernelEx(&cfg, kern, ta, tb, td, g), op, "cudaLaunchKernelEx"))
    return false;
  return check_launch(op);
}

// Whether NNC_CUDA_GEMM_PAIR (default on) lets large TF32 problems use CTA pairs.
bool gemm_pair_enabled() {
  static const bool on = [] {
    const char* e = getenv("NNC_CUDA_GEMM_PAIR");
    return !(e && e[0] == '0');
  }();
  return on;
}

void launch_simt(const Problem& p, const char* op) {
  SimtArgs a;
  a.M = p.M;
  a.N = p.N;
  a.K = p.K;
  a.batches = p.batches;
  a.A = p.A;
  a.sam = p.a_trans ? 1 : p.K;
  a.sak = p.a_trans ? p.M : 1;
  a.a_bs = p.a_bs;
  a.B = p.B;
  a.sbk = p.b_kmajor ? 1 : p.N;
  a.sbn = p.b_kmajor ? p.K : 1;
  a.b_bs = p.b_bs;
  a.alpha = p.alpha;
  a.beta = p.beta;
  a.C = p.C;
  a.c_mode = p.c_mode;
  a.ldc = p.ldc;
  a.c_bs = p.c_bs;
  a.D = p.D;
  a.ldd = p.N;
  a.d_bs = p.d_bs;
  a.relu = p.relu;
  const int64_t tiles = (int64_t)p.batches * cdiv(p.M, 16) * cdiv(p.N, 16);
  const int grid = (int)(tiles < (int64_t)sm_count() * 8 ? tiles : (int64_t)sm_count() * 8);
  gemm_simt_kernel<<<grid, 256, 0, ctx().stream>>>(a);
  check_launch(op);
}

// Splits `total / mat` matrices of `mat` elements, read at src + b * in_bs
// (in_bs == 0: one matrix), into dense hi / lo planes.
bool split_batches(const float* src, int64_t in_bs, float* hi, float* lo, int64_t mat,
                   int64_t total, const char* op) {
  split_tf32_kernel<<<grid_for(total, 256, 8), 256, 0, ctx().stream>>>(
      src, in_bs ? in_bs : mat, hi, lo, mat, total);
  return check_launch(op);
}

// Whether a problem runs on the tensor-core kernels (else the SIMT kernel).
// TMA needs 16-byte aligned bases, row pitches and batch strides. The
// reference's batch offsets (see matmul_impl) may overlap; the tensor maps
// take the batch strides as given (overlapping reads are fine).
bool tensor_core_eligible(const Problem& p) {
  const bool tiny = p.M < 64 || p.N < 16 || (int64_t)p.M * p.N * p.K < (1 << 18);
  const bool tma_ok = (p.K % 4 == 0) && aligned16(p.A) && aligned16(p.B) && (p.a_bs % 4 == 0) &&
                      p.K > 0;
  return !tiny && tma_ok;
}

void run_problem(Problem p, const char* op) {
  if ((int64_t)p.M * p.N * p.batches == 0) return;
  if (!tensor_core_eligible(p)) {
    launch_simt(p, op);
    return;
  }
  const bool split = ctx().precision == NNC_CUDA_PRECISION_3XTF32;
  // Scratch: a K-major copy of a transposed A (and of a [K, N] B that cannot
  // be read MN-major), then hi/lo planes.
  const int64_t a_elems = (int64_t)(p.a_bs ? p.batches : 1) * p.M * p.K;
  const int64_t b_elems = (int64_t)(p.b_bs ? p.batches : 1) * p.N * p.K;
  size_t need = 0;
  if (p.a_trans) need += a_elems * 4;
  if (!p.b_kmajor && !(p.N % 4 == 0 && p.b_bs % 4 == 0)) need += b_elems * 4;
  if (split) need += 2 * (a_elems + b_elems) * 4;
  float* ws = need ? (float*)workspace(need + 64, op) : nullptr;
  if (need && !ws) return;
  float* cur = ws;
  const float* A = p.A;
  const float* B = p.B;
  if (p.a_trans) {  // [K, M] -> [M, K], batches made dense
    if (!batched_transpose_f32(A, cur, p.a_bs ? p.batches : 1, p.K, p.M, op, p.a_bs)) return;
    A = cur;
    cur += a_elems;
    if (p.a_bs) p.a_bs = (int64_t)p.M * p.K;
  }
  // B stored [K, N] is read MN-major straight from its rows when they and its
  // batches start on 16-byte boundaries; otherwise it is transposed first.
  const bool b_mn = !p.b_kmajor && p.N % 4 == 0 && p.b_bs % 4 == 0;
  if (!p.b_kmajor && !b_mn) {  // [K, N] -> [N, K], batches made dense
    if (!batched_transpose_f32(B, cur, p.b_bs ? p.batches : 1, p.K, p.N, op, p.b_bs)) return;
    B = cur;
    cur += b_elems;
    if (p.b_bs) p.b_bs = (int64_t)p.N * p.K;
    p.b_kmajor = true;
  }
  const int64_t a_in_bs = p.a_bs, b_in_bs = p.b_bs;
  if (split) {  // the hi/lo planes are dense copies
    if (p.a_bs) p.a_bs = (int64_t)p.M * p.K;
    if (p.b_bs) p.b_bs = (int64_t)p.N * p.K;
  }
  if (p.softmax) {
    // Row softmax in the epilogue: every row's N <= 128 columns in one tile.
    if (split) {
      float* a_hi = cur;
      float* a_lo = a_hi + a_elems;
      float* b_hi = a_lo + a_elems;
      float* b_lo = b_hi + b_elems;
      if (!split_batches(A, a_in_bs, a_hi, a_lo, (int64_t)p.M * p.K, a_elems, op) ||
          !split_batches(B, b_in_bs, b_hi, b_lo, (int64_t)p.N * p.K, b_elems, op))
        return;
      if (p.N > 64)
        launch_tc<128, 2, 3>(p, a_hi, a_lo, b_hi, b_lo, op);
      else
        launch_tc<64, 2, 4>(p, a_hi, a_lo, b_hi, b_lo, op);
    } else if (p.N > 64) {
      launch_tc<128, 1, 6>(p, A, nullptr, B, nullptr, op);
    } else {
      launch_tc<64, 1, 8>(p, A, nullptr, B, nullptr, op);
    }
    return;
  }
  if (!split) {
    // CTA pairs: N > 128, whole 256-row tiles' worth of M, TMA-storable D and
    // enough pair tiles to keep most pairs busy.
    const bool d_tma = (p.N % 4 == 0) && (p.d_bs % 4 == 0) && aligned16(p.D);
    if (gemm_pair_enabled() && d_tma && p.N > 128 && p.M >= 2 * BM &&
        (int64_t)cdiv(p.M, 2 * BM) * cdiv(p.N, 256) * p.batches >= sm_count() / 2 - 10) {
      launch_tc2<256, 6>(p, A, B, op);
      return;
    }
    // Batched A of at most 128 rows per batch against one B: each pair takes
    // two consecutive batches (one per CTA) and splits B's tile between them.
    if (gemm_pair_enabled() && d_tma && p.N > 128 && p.M <= BM && p.a_bs != 0 && p.b_bs == 0 &&
        p.batches >= 2 && (int64_t)(p.batches + 1) / 2 * cdiv(p.N, 256) >= sm_count() / 2 - 10) {
      launch_tc2<256, 6>(p, A, B, op, true);
      return;
    }
    if (p.N > 128 && (int64_t)cdiv(p.M, BM) * cdiv(p.N, 256) * p.batches >= sm_count())
      launch_tc<256, 1, 4>(p, A, nullptr, B, nullptr, op);
    else if (p.N > 64)
      launch_tc<128, 1, 6>(p, A, nullptr, B, nullptr, op);
    else
      launch_tc<64, 1, 8>(p, A, nullptr, B, nullptr, op);
    return;
  }
  float* a_hi = cur;
  float* a_lo = a_hi + a_elems;
  float* b_hi = a_lo + a_elems;
  float* b_lo = b_hi + b_elems;
  if (!split_batches(A, a_in_bs, a_hi, a_lo, (int64_t)p.M * p.K, a_elems, op) ||
      !split_batches(B, b_in_bs, b_hi, b_lo, (int64_t)p.N * p.K, b_elems, op))
    return;
  if (p.N > 64)
    launch_tc<128, 2, 3>(p, a_hi, a_lo, b_hi, b_lo, op);
  else
    launch_tc<64, 2, 4>(p, a_hi, a_lo, b_hi, b_lo, op);
}

bool f32(const Tensor* t, const char* op, const char* name) {
  if (!valid_tensor(t, op, name)) return false;
  if (elem_type(t) != NNC_DTYPE_FLOAT32 || tag_of(t) != 0) {
    fail(NNC_CUDA_ERR_UNSUPPORTED, op, "%s: needs an untagged float32 tensor", name);
    return false;
  }
  return true;
}

bool set_c(Problem& p, Tensor* c, int M, int N, const char* op) {
  p.C = nullptr;
  p.c_mode = 0;
  p.ldc = N;
  p.c_bs = 0;
  if (!c) return true;
  if (!f32(c, op, "c")) return false;
  p.C = (const float*)c->data;
  if (c->ndim == 1) {
    if (numel(c) < N) {
      fail(NNC_CUDA_ERR_INVALID, op, "c has %lld elements, needs %d", (long long)numel(c), N);
      return false;
    }
    p.c_mode = 1;
  } else {
    if (numel(c) < (int64_t)M * N) {
      fail(NNC_CUDA_ERR_INVALID, op, "c has %lld elements, needs %lld", (long long)numel(c),
           (long long)M * N);
      return false;
    }
    p.c_mode = 2;
  }
  return true;
}

// nnc_gemm semantics (ops.c:1732-1841).
void gemm_impl(Tensor* a, Tensor* b, Tensor* c, Tensor* out, float alpha, float beta,
               int trans_a, int trans_b, int relu, const char* op) {
  OpScope scope(op);
  if (!f32(a, op, "a") || !f32(b, op, "b") || !f32(out, op, "output")) return;
  trace_io(tensor_bytes(a) + tensor_bytes(b) + tensor_bytes(c), tensor_bytes(out));
  int M, N, K;
  if (a->ndim == 2 && b->ndim == 2) {
    M = (int)(trans_a ? a->shape[1] : a->shape[0]);
    K = (int)(trans_a ? a->shape[0] : a->shape[1]);
    N = (int)(trans_b ? b->shape[0] : b->shape[1]);
    const int kb = (int)(trans_b ? b->shape[1] : b->shape[0]);
    if (kb != K) {
      fail(NNC_CUDA_ERR_INVALID, op, "inner dimensions differ (%d vs %d)", K, kb);
      return;
    }
  } else if (a->ndim == 1 && b->ndim == 2) {
    M = 1;
    K = (int)a->shape[0];
    N = (int)b->shape[1];
    trans_a = 0;  // N = b->shape[1] even when trans_b is set, as ops.c:1779-1784
  } else if (a->ndim == 2 && b->ndim == 1) {
    M = (int)a->shape[0];
    K = (int)a->shape[1];
    N = 1;
    trans_b = 0;
  } else {
    M = 1;
    K = (int)numel(a);
    N = (int)numel(b);
    trans_a = 0;
    trans_b = 0;
  }
  if (numel(out) < (int64_t)M * N || numel(a) < (int64_t)M * K || numel(b) < (int64_t)K * N) {
    fail(NNC_CUDA_ERR_INVALID, op, "operand sizes do not cover M=%d N=%d K=%d", M, N, K);
    return;
  }
  Problem p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.batches = 1;
  p.A = (const float*)a->data;
  p.a_trans = trans_a != 0;
  p.B = (const float*)b->data;
  p.b_kmajor = trans_b != 0;
  p.alpha = alpha;
  p.beta = beta;
  p.D = (float*)out->data;
  p.relu = relu;
  if (!set_c(p, c, M, N, op)) return;
  run_problem(p, op);
}

// nnc_gemm_nt semantics (ops.c:1843-1886): B stored [N, K]. The body, for
// callers that have opened the call's scope themselves.
void gemm_nt_body(Tensor* a, Tensor* b, Tensor* c, Tensor* out, float alpha, float beta, int relu,
                  const char* op);
void gemm_nt_impl(Tensor* a, Tensor* b, Tensor* c, Tensor* out, float alpha, float beta, int relu,
                  const char* op) {
  OpScope scope(op);
  if (!f32(a, op, "a") || !f32(b, op, "b") || !f32(out, op, "output")) return;
  trace_io(tensor_bytes(a) + tensor_bytes(b) + tensor_bytes(c), tensor_bytes(out));
  gemm_nt_body(a, b, c, out, alpha, beta, relu, op);
}
void gemm_nt_body(Tensor* a, Tensor* b, Tensor* c, Tensor* out, float alpha, float beta, int relu,
                  const char* op) {
  int M, N, K;
  if (a->ndim == 2 && b->ndim == 2) {
    M = (int)a->shape[0];
    K = (int)a->shape[1];
    N = (int)b->shape[0];
  } else if (a->ndim == 1 && b->ndim == 2) {
    M = 1;
    K = (int)a->shape[0];
    N = (int)b->shape[0];
  } else {
    M = 1;
    K = (int)numel(a);
    N = (b->ndim == 2) ? (int)b->shape[0] : (int)numel(b);
  }
  if (numel(out) < (int64_t)M * N) {
    fail(NNC_CUDA_ERR_INVALID, op, "output too small");
    return;
  }
  Problem p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.batches = 1;
  p.A = (const float*)a->data;
  p.B = (const float*)b->data;
  p.b_kmajor = true;
  p.alpha = alpha;
  p.beta = beta;
  p.D = (float*)out->data;
  p.relu = relu;
  if (!set_c(p, c, M, N, op)) return;
  run_problem(p, op);
}

// nnc_matmul semantics (ops.c:1607-1730), optional bias (row broadcast) + relu.
// nnc_matmul and its fused forms: D = alpha * A B (+ bias[n]) (relu), or the
// softmax of alpha * A B over the last axis.
void matmul_impl(Tensor* a, Tensor* b, Tensor* bias, Tensor* out, int relu, const char* op,
                 float alpha = 1.0f, bool softmax = false) {
  OpScope scope(op);
  if (!f32(a, op, "a") || !f32(b, op, "b") || !f32(out, op, "output")) return;
  trace_io(tensor_bytes(a) + tensor_bytes(b) + tensor_bytes(bias), tensor_bytes(out));
  Problem p{};
  p.alpha = alpha;
  p.beta = 1.0f;
  p.A = (const float*)a->data;
  p.B = (const float*)b->data;
  p.D = (float*)out->data;
  p.relu = relu;
  p.batches = 1;
  if (a->ndim == 2 && b->ndim == 2) {
    p.M = (int)a->shape[0];
    p.K = (int)a->shape[1];
    p.N = (int)b->shape[1];
  } else if (a->ndim == 1 && b->ndim == 2) {
    p.M = 1;
    p.K = (int)a->shape[0];
    p.N = (int)b->shape[1];
  } else if (a->ndim == 2 && b->ndim == 1) {
    p.M = (int)a->shape[0];
    p.K = (int)a->shape[1];
    p.N = 1;
  } else if (a->ndim >= 2 && b->ndim >= 2) {
    const int od = out->ndim;
    int64_t batch = 1;
    for (int i = 0; i < od - 2; ++i) batch *= out->shape[i];
    p.M = (int)out->shape[od - 2];
    p.N = (int)out->shape[od - 1];
    p.K = (int)a->shape[a->ndim - 1];
    // Batch offsets exactly as ops.c:1686-1708 computes them: the offset of
    // batch i in `a` is i * (numel(a) / (M_a * K)) elements — the number of
    // matrices in a, not their size — and likewise for b unless b has fewer
    // dims than the output (then offset 0). Output batches are dense (M * N).
    p.a_bs = numel(a) / (a->shape[a->ndim - 2] * a->shape[a->ndim - 1]);
    p.b_bs = (b->ndim < od) ? 0 : numel(b) / (b->shape[b->ndim - 2] * b->shape[b->ndim - 1]);
    if (batch == 1) {
      p.a_bs = 0;
      p.b_bs = 0;
    }
    p.batches = (int)batch;
    p.d_bs = (int64_t)p.M * p.N;
  } else {
    fail(NNC_CUDA_ERR_UNSUPPORTED, op, "unsupported ranks (%d, %d)", a->ndim, b->ndim);
    return;
  }
  if (numel(out) < (int64_t)p.M * p.N * p.batches) {
    fail(NNC_CUDA_ERR_INVALID, op, "output too small");
    return;
  }
  p.b_kmajor = false;
  p.C = nullptr;
  p.c_mode = 0;
  p.ldc = p.N;
  if (bias) {
    if (!f32(bias, op, "bias")) return;
    if (numel(bias) < p.N) {
      fail(NNC_CUDA_ERR_INVALID, op, "bias shorter than N");
      return;
    }
    p.C = (const float*)bias->data;
    p.c_mode = 1;
  }
  if (softmax) {
    // Fused into the epilogue when every row fits one tensor-core tile;
    // otherwise the contraction, then the row softmax in place.
    if (tensor_core_eligible(p) && p.N <= 128) {
      p.softmax = 1;
    } else {
      run_problem(p, op);
      if (ctx().status == NNC_CUDA_OK) nnc_softmax(out, out, -1);
      return;
    }
  }
  run_problem(p, op);
}

}  // namespace
}  // namespace nnc

using namespace nnc;

extern "C" {

void nnc_gemm(Tensor* a, Tensor* b, Tensor* c, Tensor* output, float alpha, float beta,
              int trans_a, int trans_b) {
  gemm_impl(a, b, c, output, alpha, beta, trans_a, trans_b, 0, "nnc_gemm");
}
void nnc_gemm_relu(Tensor* a, Tensor* b, Tensor* c, Tensor* output, float alpha, float beta,
                   int trans_a, int trans_b) {
  gemm_impl(a, b, c, output, alpha, beta, trans_a, trans_b, 1, "nnc_gemm_relu");
}
void nnc_gemm_nt(Tensor* a, Tensor* b, Tensor* c, Tensor* output, float alpha, float beta) {
  gemm_nt_impl(a, b, c, output, alpha, beta, 0, "nnc_gemm_nt");
}
void nnc_gemm_nt_relu(Tensor* a, Tensor* b, Tensor* c, Tensor* output, float alpha, float beta) {
  gemm_nt_impl(a, b, c, output, alpha, beta, 1, "nnc_gemm_nt_relu");
}

// GlobalAveragePool -> Flatten -> Gemm(transB = 1) as one call: the pooled
// [N, C] features go to the end of the workspace (whose front holds what the
// GEMM itself may need: the 3xTF32 hi/lo planes of both operands), never to
// an arena tensor, and no flatten copy runs. Same arithmetic as
// nnc_avgpool2d(kernel = stride = H x W) then nnc_gemm_nt.
void nnc_gap_gemm_nt(Tensor* input, Tensor* b, Tensor* c, Tensor* output, float alpha,
                     float beta) {
  const char* op = "nnc_gap_gemm_nt";
  OpScope scope(op);
  // The pooled input may be channels-last (tagged); the GEMM operands not.
  if (!valid_tensor(input, op, "input") || !f32(b, op, "b") || !f32(output, op, "output")) return;
  if (elem_type(input) != NNC_DTYPE_FLOAT32 || (tag_of(input) & ~NNC_CUDA_TAG_NHWC) != 0) {
    fail(NNC_CUDA_ERR_UNSUPPORTED, op, "input: needs a float32 tensor (NCHW or channels-last)");
    return;
  }
  if (input->ndim != 4 || b->ndim != 2 || input->shape[1] != b->shape[1]) {
    fail(NNC_CUDA_ERR_INVALID, op, "expected a 4-D input [N, C, H, W] and b [O, C]");
    return;
  }
  trace_io(tensor_bytes(input) + tensor_bytes(b) + tensor_bytes(c), tensor_bytes(output));
  const int64_t N = input->shape[0], C = input->shape[1], O = b->shape[0];
  const int H = (int)input->shape[2], W = (int)input->shape[3];
  const bool split = ctx().precision == NNC_CUDA_PRECISION_3XTF32;
  const size_t front = ((split ? 2 * (size_t)(N * C + O * C) * 4 : 0) + 64 + 255) & ~(size_t)255;
  char* ws = (char*)workspace(front + (size_t)N * C * 4, op);
  if (!ws) return;
  float* pooled = (float*)(ws + front);
  if (!launch_avgpool_f32((const float*)input->data, pooled, (int)N, (int)C, H, W, 1, 1, H, W, H, W,
                          0, 0, is_nhwc(input), op))
    return;
  int64_t shape[2] = {N, C};
  Tensor flat{pooled, NNC_DTYPE_FLOAT32, shape, 2, N * C * 4};
  gemm_nt_body(&flat, b, c, output, alpha, beta, 0, op);
}
void nnc_matmul(Tensor* a, Tensor* b, Tensor* output) {
  matmul_impl(a, b, nullptr, output, 0, "nnc_matmul");
}
void nnc_matmul_bias(Tensor* a, Tensor* b, Tensor* bias, Tensor* output) {
  matmul_impl(a, b, bias, output, 0, "nnc_matmul_bias");
}
void nnc_matmul_scale_softmax(Tensor* a, Tensor* b, Tensor* output, float alpha) {
  matmul_impl(a, b, nullptr, output, 0, "nnc_matmul_scale_softmax", alpha, true);
}
void nnc_matmul_relu(Tensor* a, Tensor* b, Tensor* bias, Tensor* output) {
  matmul_impl(a, b, bias, output, 1, "nnc_matmul_relu");
}

}  // extern "C"
