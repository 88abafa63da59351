// Shared host/device helpers of libnnc_cuda.so: tensor metadata, status
// reporting, the per-thread execution context and launch checking.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include "nnc_cuda.h"
#include "nnc_ops.h"

namespace nnc {

// ---------------------------------------------------------------------------
// Per-thread execution context (device, stream, precision, sticky status).
// ---------------------------------------------------------------------------
struct ThreadCtx {
  int device = 0;
  cudaStream_t stream = nullptr;
  int precision = NNC_CUDA_PRECISION_TF32;
  int status = NNC_CUDA_OK;
  char message[512] = {0};
  long long launches = 0;
};
ThreadCtx& ctx();

// Records a failure: sets the sticky status, keeps the first message and
// prints one line to stderr (the reference prints and returns on invalid
// tensors, ops.c:728-744).
void fail(int code, const char* op, const char* fmt, ...)
    __attribute__((format(printf, 3, 4)));

// Checks the result of a launch / runtime call; false (and status set) on error.
bool check_cuda(cudaError_t err, const char* op, const char* what);
// Call once right after every kernel launch: checks it and counts it.
inline bool check_launch(const char* op) {
  ++ctx().launches;
  return check_cuda(cudaGetLastError(), op, "kernel launch");
}

// Device-side error word of the current device (bounded waits that expire
// set it to NNC_CUDA_ERR_DEVICE_TIMEOUT; the host reads it on demand).
int* device_error_word();
int sm_count();
// True once the current device's state (error word, SM count) exists, so
// that device_error_word() and sm_count() allocate nothing; nnc_cuda_init
// creates it. Never allocates.
bool device_ready();

// Scratch memory on the current device for the current stream.
void* workspace(size_t bytes, const char* op);

// Stream-K scratch on the current device for this thread: `slots` partial
// slots of slot_bytes each and one zeroed arrival counter per slot. Returns
// false, recording no error, when it cannot be had without allocating inside
// a graph capture or beside a caller-supplied workspace (or the allocation
// fails): the caller then runs without stream-K. Like the workspace, it is
// shared by the thread's calls, which must therefore run in stream order.
constexpr size_t kStreamKCounterBytes = 4096;
bool streamk_scratch(int slots, size_t slot_bytes, unsigned** counters, float** parts);

// Max / average pooling between two device buffers (pool.cu), nnc_maxpool2d /
// nnc_avgpool2d semantics.
bool launch_maxpool_f32(const float* in, float* out, int N, int C, int H, int W, int OH, int OW,
                        int kh, int kw, int sh, int sw, int ph, int pw, bool nhwc, const char* op);
bool launch_avgpool_f32(const float* in, float* out, int N, int C, int H, int W, int OH, int OW,
                        int kh, int kw, int sh, int sw, int ph, int pw, bool nhwc, const char* op);

// Opened at the top of every entry point: refreshes the thread's device from
// the CUDA runtime (so callers that switch devices with cudaSetDevice or
// torch.cuda.set_device are followed) and, when tracing is enabled
// (nnc_cuda_trace_enable / NNC_CUDA_TRACE=1), brackets the call's launches
// with CUDA events on the current stream.
struct OpScope {
  explicit OpScope(const char* name);
  ~OpScope();
  const char* name_;
  int slot_;
  int prev_slot_;
  bool prev_captured_;
};
// Bytes of a tensor's storage (nbytes, else numel x element size; 0 for NULL).
uint64_t tensor_bytes(const Tensor* t);
// Records on the innermost open OpScope of this thread (when it is traced)
// the bytes of the tensors the call reads and writes (the trace's in= / out=);
// a call's first annotation stands.
void trace_io(uint64_t in_bytes, uint64_t out_bytes);

// ---------------------------------------------------------------------------
// Tensor metadata helpers (host).
// ---------------------------------------------------------------------------
inline int elem_type(const Tensor* t) { return (int)t->dtype & NNC_CUDA_DTYPE_MASK; }
inline int tag_of(const Tensor* t) { return (int)t->dtype & ~NNC_CUDA_DTYPE_MASK; }
inline bool is_nhwc(const Tensor* t) { return (tag_of(t) & NNC_CUDA_TAG_NHWC) != 0; }
inline size_t elem_size(int dtype) {
  switch (dtype) {
    case NNC_DTYPE_FLOAT16: return 2;
    case NNC_DTYPE_INT8:
    case NNC_DTYPE_UINT8:
    case NNC_DTYPE_BOOL: return 1;
    case NNC_DTYPE_INT64: return 8;
    default: return 4;
  }
}
// Product of the extents (the reference's tensor_numel, ops.c:22-28).
inline int64_t numel(const Tensor* t) {
  int64_t n = 1;
  for (int i = 0; i < t->ndim; ++i) n *= t->shape[i];
  return n;
}
// NULL checks shared by every entry point.
bool valid_tensor(const Tensor* t, const char* op, const char* name);
inline bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

// ---------------------------------------------------------------------------
// Programmatic dependent launch. Kernels on the forward path are launched
// with the programmatic-stream-serialisation attribute (captured into CUDA
// graphs as programmatic edges): each kernel lets the next one be scheduled
// as soon as all of its own CTAs have started (pdl_trigger, first thing), and
// the next one's CTAs run their prologue (barrier set-up, TMEM allocation,
// tensor-map prefetch) on SMs freed by the tail of this one, then wait
// (pdl_wait) until this grid has completed and its writes are visible before
// touching any activation memory (reads, and writes to arena slots the
// previous kernel may still read). Launched without the attribute, both are
// no-ops. NNC_CUDA_PDL=0 turns the attribute off.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
bool pdl_enabled();

// Launches `kern` on the current stream with the PDL attribute (when
// enabled), like `kern<<<grid, block, smem, stream>>>(args...)`: follow it
// with check_launch(op), which counts it and checks the launch.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = ctx().stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

// Grid for a kernel whose blocks loop over `work` units: every block
// resident at once (the occupancy of `kern` at this block size, per device,
// cached), or `work` blocks when there are fewer. A grid between the two
// leaves its last blocks waiting until whole loops of others end.
template <typename K>
int resident_grid(K kern, int threads, size_t smem, int64_t work) {
  static int per_sm[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  int& r = per_sm[dev & 63];
  if (r == 0) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&r, kern, threads, smem) != cudaSuccess || r <= 0) {
      cudaGetLastError();
      r = 1;
    }
  }
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = 148;
  const int64_t cap = (int64_t)sms * r;
  return (int)(work < cap ? (work < 1 ? 1 : work) : cap);
}

// Ceil-div and grid sizing in multiples of the SM count.
__host__ __device__ inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }
int grid_for(int64_t work_items, int threads, int max_ctas_per_sm = 8);

}  // namespace nnc
