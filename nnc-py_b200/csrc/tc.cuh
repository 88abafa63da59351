// sm_100a building blocks for the tensor-core kernels: mbarriers with bounded
// waits, TMA tiled loads (no multicast), tcgen05 TMEM allocation, MMA,
// commit and loads, and the host-side tensor-map encoder.
//
// Every wait is bounded: after kWaitLimit polls the waiting thread records
// NNC_CUDA_ERR_DEVICE_TIMEOUT in the device error word and returns false, so
// a broken pipeline ends the kernel instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace nnc {
namespace tc {

constexpr uint32_t kWaitLimit = 1u << 24;  // tries; the 2 s time bound ends a wait first

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------- mbarrier --
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
// One try with a suspend-time hint: a thread whose phase has not completed
// sleeps in hardware until it does or kSuspendNs pass, instead of spinning
// and taking issue slots from the warps that do the work.
#ifndef NNC_MBAR_SUSPEND_NS
#define NNC_MBAR_SUSPEND_NS 100000  // 0.1 ms per try
#endif
constexpr uint32_t kSuspendNs = NNC_MBAR_SUSPEND_NS;
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  if constexpr (kSuspendNs == 0) {  // the system-dependent time limit
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendNs)
        : "memory");
  }
  return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait for the phase with the given parity to complete: suspending
// tries until it does, giving up after kWaitNs nanoseconds (or kWaitLimit
// tries) and recording the timeout.
constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s
__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity, int* err,
                                              uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (global_ns() - t0 > limit_ns) break;
  }
  if (err) atomicExch(err, 5 /* NNC_CUDA_ERR_DEVICE_TIMEOUT */);
  return false;
}
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  return mbar_wait_for(bar, parity, err, kWaitNs);
}

// ---------------------------------------------------------------- TMA ----
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}
// TMA store of a 3-D box from shared memory (bulk-group completion). The
// box's x coordinate times the element size must be a multiple of 16 bytes
// and no coordinate may be negative; parts of the box outside the tensor are
// not written.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int x,
                                             int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
      : "memory");
}
__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Waits until at most N committed bulk groups still read their shared source.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Waits until at most N committed bulk groups are incomplete.
template <int N>
__device__ __forceinline__ void bulk_wait_group() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}
// Untiled bulk copies (no tensor map): both addresses 16-byte aligned, the
// size a multiple of 16 bytes. The load completes `bytes` on the mbarrier;
// the store joins the current bulk group.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void bulk_store(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(
                   reinterpret_cast<uint64_t>(dst)),
               "r"(smem_u32(src)), "r"(bytes)
               : "memory");
}
// Makes this thread's generic-proxy shared-memory writes visible to the
// async proxy (a following TMA store reads them).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y, int z, int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}
// im2col load over an NHWC tensor map: starts at pixel (w, h, n) of the map's
// bounding box (which must be a real output pixel's window origin) and walks
// pixelsPerColumn pixels along W, H, N; (ow, oh) is the filter-tap offset
// added to every pixel; channels [c, c + channelsPerPixel).
__device__ __forceinline__ void tma_load_im2col_4d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                                   int c, int w, int h, int n, uint16_t ow,
                                                   uint16_t oh) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.im2col.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2], {%7, %8};" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c), "r"(w), "r"(h), "r"(n),
      "h"(ow), "h"(oh)
      : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ------------------------------------------------------------ tcgen05 ----
// TMEM allocation (one full warp executes these).
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::tf32, issued by one thread.
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on `bar` once all previously issued MMAs of this thread complete.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// One lane of the (fully active) warp returns true: the MMA loops run on the
// whole warp so their operands stay warp-uniform, and the elected lane issues.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b32 r;\n\t"
      "elect.sync r|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}
// mbar_wait by every lane of a warp; false on every lane if any lane timed out.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, int* err) {
  const bool ok = mbar_wait(bar, parity, err);
  return __all_sync(0xffffffffu, ok);
}

// 32 lanes x 32 bit, 16 consecutive columns: thread i of the warp receives
// TMEM lane (addr.lane + i), columns [addr.col, addr.col + 16).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32"
      " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// 16 lanes x 256 bits, 4 repetitions (32 columns): thread t receives, for
// repetition q, lane (t >> 2) at columns 8q + 2 (t & 3) + {0, 1} in r[4q],
// r[4q + 1] and lane (t >> 2) + 8 at the same columns in r[4q + 2], r[4q + 3].
__device__ __forceinline__ void tmem_ld_16x256b_x4(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x4.b32"
      " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// The same shape with 2 repetitions (16 columns): r[4q .. 4q + 3], q = 0, 1.
__device__ __forceinline__ void tmem_ld_16x256b_x2(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.16x256b.x2.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                 "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// Stores 16 consecutive 32-bit columns of this warp's 32 TMEM lanes (lane i
// of the warp writes lane base + i).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32"
      " [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Chunked accumulation of the 3xTF32 contractions. Measured on B200, the
// error of a K-long 3xTF32 dot product accumulated in one TMEM accumulator
// grows ~K^1.5 (normwise 8e-6 at K = 2048, 3.4e-5 at 8192): the accumulator
// does not round to nearest, and its error follows the running sum. So the
// MMA issuer restarts the accumulator every kChunkKBlocks k-blocks in
// alternating TMEM buffers, and the epilogue warps fold each chunk's partial
// sums into a running sum held in TMEM with round-to-nearest fp32 adds.
// promote_chunk32 does that for one warp's 32 lanes x 32 columns: `part` is
// the chunk's buffer column, `sum` the running sum's; the first chunk copies,
// later ones add; the last chunk writes the total back over its own buffer,
// where the tile's ordinary epilogue reads it. The caller waits for the
// stores (tmem_st_wait) before releasing the buffer. A single-chunk
// reduction needs no call.
constexpr int kChunkKBlocks = 4;  // k-blocks of 32 (K = 128) per chunk
__device__ __forceinline__ void promote_chunk32(uint32_t lane_addr, uint32_t part, uint32_t sum,
                                                bool first, bool last) {
  const uint32_t dst = lane_addr + (last ? part : sum);
#pragma unroll 1
  for (uint32_t h = 0; h < 32; h += 8) {  // 8 columns at a time (register budget)
    uint32_t p[8], q[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(p[0]), "=r"(p[1]), "=r"(p[2]), "=r"(p[3]), "=r"(p[4]), "=r"(p[5]),
                   "=r"(p[6]), "=r"(p[7])
                 : "r"(lane_addr + part + h));
    if (!first)
      asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                   : "=r"(q[0]), "=r"(q[1]), "=r"(q[2]), "=r"(q[3]), "=r"(q[4]), "=r"(q[5]),
                     "=r"(q[6]), "=r"(q[7])
                   : "r"(lane_addr + sum + h));
    tmem_ld_wait();
    if (!first) {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        p[j] = __float_as_uint(__fadd_rn(__uint_as_float(q[j]), __uint_as_float(p[j])));
    }
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(
                     dst + h),
                 "r"(p[0]), "r"(p[1]), "r"(p[2]), "r"(p[3]), "r"(p[4]), "r"(p[5]), "r"(p[6]),
                 "r"(p[7])
                 : "memory");
  }
}

// Shared-memory matrix descriptor: K-major operand in the 128-byte swizzle
// layout written by TMA with CU_TENSOR_MAP_SWIZZLE_128B (rows of 128 bytes,
// 8-row groups 1024 bytes apart). Fields: start address >> 4 [0,14),
// leading byte offset >> 4 [16,30) (unused for swizzled K-major, 1),
// stride byte offset >> 4 [32,46) = 1024 >> 4, version 1 at bit 46,
// layout type SWIZZLE_128B = 2 at [61,64).
__device__ __forceinline__ uint64_t desc_kmajor_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr & 0x3FFFFu) >> 4);
  d |= (uint64_t)1u << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}

// K-major operand in the 128-byte (row_bytes 128, layout type 2) or 64-byte
// (row_bytes 64, layout type 4) swizzle layout with a caller-chosen distance
// between 8-row groups (a multiple of row_bytes): rows of a group are
// consecutive rows, and the swizzle phase follows the absolute address, so a
// group may start at any row (measured on sm_100a for both spans, with the
// base-offset field left 0).
__device__ __forceinline__ uint64_t desc_kmajor_swz(uint32_t smem_addr, uint32_t sbo,
                                                    int row_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr & 0x3FFFFu) >> 4);
  d |= (uint64_t)1u << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)(row_bytes == 64 ? 4u : 2u) << 61;
  return d;
}

// Shared-memory matrix descriptor: K-major operand without swizzling, made of
// 8-row x 16-byte core matrices stored contiguously (128 bytes each): core
// matrices adjacent along M are `sbo` bytes apart, along K `lbo` bytes apart.
__device__ __forceinline__ uint64_t desc_kmajor_noswizzle(uint32_t smem_addr, uint32_t lbo,
                                                          uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;
  return d;  // layout type 0 = SWIZZLE_NONE
}

// Shared-memory matrix descriptor: MN-major fp32 operand in the 128-byte,
// 32-byte-atom swizzle (layout type 1, the only MN-major layout kind::tf32
// accepts), as TMA writes a {32 (MN), rows (K)} box with
// CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B: each 128-byte row holds 32
// consecutive MN elements of one k, 4-k groups are 512 bytes apart (stride
// byte offset) and successive 32-element MN chunks are `lbo` bytes apart
// (leading byte offset). One MMA (K = 8) reads two 4-row groups per chunk.
__device__ __forceinline__ uint64_t desc_mn_sw128_atom32(uint32_t smem_addr, uint32_t lbo) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)(512u >> 4) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)1u << 61;
  return d;
}

// Instruction-descriptor bit that marks the B operand MN-major ("transpose B").
constexpr uint32_t kIdescBMajorMN = 1u << 16;

// Instruction descriptor for kind::tf32 with fp32 accumulation, both operands
// K-major: c_format F32 (1) at [4,6), a/b_format TF32 (2) at [7,10)/[10,13),
// N >> 3 at [17,23), M >> 4 at [24,29).
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

// Round an fp32 value to the nearest TF32 value (ties away from zero); the
// result has its 13 low mantissa bits clear.
__device__ __forceinline__ float to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// ------------------------------------------------- CTA pairs (2-SM MMA) ----
// A cluster of two CTAs sharing one M = 256 tile: the even CTA issues
// tcgen05.mma.cta_group::2 for both, each CTA holding its 128 rows of A, its
// half of B's rows and its 128 TMEM lanes of the accumulator. No TMA load
// here uses cluster multicast; commits may signal both CTAs' barriers.
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// The shared::cluster address of `smem_addr` (a shared::cta address of this
// CTA) in the shared memory of cluster CTA `rank`.
__device__ __forceinline__ uint32_t mapa(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}
// Every thread of both CTAs: release this CTA's prior shared-memory writes
// (barrier inits included) to the pair and wait for the peer.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" :::
                   "memory");
}
// Pair TMEM allocation: one warp of each CTA executes these together.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
// D (+)= A * B^T over the pair, kind::tf32, issued by one thread of the even CTA.
__device__ __forceinline__ void mma_tf32_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                              uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on the barrier at `bar`'s offset in both CTAs of the pair when
// this thread's prior pair MMAs complete.
__device__ __forceinline__ void mma_commit_pair_both(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 "
      "[%0], %1;" ::"r"(smem_u32(bar)),
      "h"((uint16_t)3)
      : "memory");
}
// Arrive on an mbarrier of another cluster CTA (a mapa address), with the
// default release at CTA scope. Its users hand a TMEM accumulator back to the
// pair's MMA issuer: the arriving warps' TMEM reads are ordered by tcgen05
// fences around the arrive and the wait, and the waiter reads nothing that
// this CTA stored to global memory, which a cluster-scope release would
// first wait for (ncu showed epilogue warps stalled on that memory barrier).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// TMA loads into this CTA's shared memory whose completion is counted on an
// mbarrier of either CTA of the pair (`bar` a shared::cluster address).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar,
                                                 int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d_pair(void* dst, const CUtensorMap* map, uint32_t bar,
                                                 int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "r"(z)
      : "memory");
}
__device__ __forceinline__ void tma_load_4d_pair(void* dst, const CUtensorMap* map, uint32_t bar,
                                                 int x, int y, int z, int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}
__device__ __forceinline__ void tma_load_im2col_4d_pair(void* dst, const CUtensorMap* map,
                                                        uint32_t bar, int c, int w, int h, int n,
                                                        uint16_t ow, uint16_t oh) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.im2col.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2], {%7, %8};" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c), "r"(w), "r"(h), "r"(n), "h"(ow),
      "h"(oh)
      : "memory");
}

}  // namespace tc

// swizzle_bytes value selecting CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B: 128-byte
// rows whose four 32-byte chunks are XOR-permuted by (row & 3), the layout
// MN-major kind::tf32 operands take (descriptor layout type 1).
constexpr int kSwizzle128Atom32 = 32;

// Host: encodes a tiled tensor map (fp32, zero OOB fill) over a row-major
// tensor with dims[0] innermost, in the 128-byte (default), 64-byte or
// 128-byte 32-byte-atom (kSwizzle128Atom32) swizzle layout (the box's inner
// extent must equal the span). Returns false
// (status set) on failure. strides_bytes has rank-1 entries (dims 1..rank-1).
bool encode_tmap_f32(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                     const uint64_t* strides_bytes, const uint32_t* box,
                     const uint32_t* elem_strides, const char* op, int swizzle_bytes = 128);

// Host: encodes a 4-D im2col tensor map (fp32, zero OOB fill) over an NHWC
// tensor: dims {C, W, H, N}, strides_bytes for W, H, N; bounding-box corners
// {lower, upper} applied to both W and H (callers only use square windows);
// elem_strides {1, stride, stride, 1}; swizzle128 selects SWIZZLE_128B (one
// 128-byte row per pixel) or SWIZZLE_NONE.
bool encode_tmap_im2col_f32(CUtensorMap* map, const void* base, const uint64_t* dims,
                            const uint64_t* strides_bytes, int lower, int upper,
                            uint32_t channels_per_pixel, uint32_t pixels_per_column,
                            uint32_t stride, bool swizzle128, const char* op);

}  // namespace nnc
