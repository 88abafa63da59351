/*
 * nnc_cuda.h — control surface of the B200 operator library (libnnc_cuda.so).
 *
 * The reference operator library (nnc-py runtime/x86/ops.c) is synchronous,
 * host-memory and stateless; its runtime header (runtime/include/
 * nnc_runtime.h:22-42) declares allocation/scheduler hooks that nothing
 * defines. On a GPU the operators need a device, a stream, a precision mode
 * for the tensor-core contractions, scratch memory and an error channel;
 * this header provides them. Everything here is extern "C" with plain
 * pointers and integers.
 *
 * State model:
 *   - device, stream, precision and the sticky error status are per host
 *     thread (a thread that never calls the setters uses device 0, the
 *     legacy default stream, TF32 precision);
 *   - scratch ("workspace") memory is per (thread, device): either supplied by
 *     the caller (nnc_cuda_set_workspace) or grown on demand with stream-ordered
 *     allocation on the current stream.
 */
#ifndef NNC_CUDA_H
#define NNC_CUDA_H

#include <stddef.h>
#include <stdint.h>

#include "nnc_types.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------------- */
#define NNC_CUDA_OK 0
#define NNC_CUDA_ERR_INVALID 1      /* NULL tensor/data/shape, shape mismatch */
#define NNC_CUDA_ERR_UNSUPPORTED 2  /* valid for the reference, not supported here */
#define NNC_CUDA_ERR_LAUNCH 3       /* CUDA runtime / launch error */
#define NNC_CUDA_ERR_NOMEM 4        /* workspace or slab allocation failed */
#define NNC_CUDA_ERR_DEVICE_TIMEOUT 5 /* a bounded in-kernel wait expired */

/* ---- storage tags carried in Tensor::dtype above the element type -------- */
#define NNC_CUDA_DTYPE_MASK 0xff
/* 4-D activation stored channels-last ([N][H][W][C]) while Tensor::shape
 * keeps the logical NCHW extents. Only the conv/pool entry points and the
 * element-wise ops accept it. */
#define NNC_CUDA_TAG_NHWC 0x100
/* Conv weight re-laid out by nnc_cuda_prepack_conv_weight. */
#define NNC_CUDA_TAG_PACKED_CONV 0x200

/* ---- precision of tcgen05 contractions (conv, gemm, matmul) -------------- */
#define NNC_CUDA_PRECISION_TF32 0   /* one TF32 MMA per k-step */
#define NNC_CUDA_PRECISION_3XTF32 1 /* hi*hi + hi*lo + lo*hi split: ~fp32 accuracy */

/* ---- device / stream / status ------------------------------------------- */
int nnc_cuda_init(int device);           /* set device + create its state */
int nnc_cuda_set_device(int device);
int nnc_cuda_get_device(void);
void nnc_cuda_set_stream(void* stream);  /* cudaStream_t; NULL = legacy default */
void* nnc_cuda_get_stream(void);
int nnc_cuda_sync(void);                 /* synchronise the current stream */
int nnc_cuda_get_last_error(void);       /* sticky per-thread status */
const char* nnc_cuda_get_last_error_string(void);
void nnc_cuda_clear_error(void);
/* Reads (and clears) the device-side error word that kernels set when a
 * bounded wait expires; synchronises the current stream first. Returns
 * NNC_CUDA_OK or NNC_CUDA_ERR_DEVICE_TIMEOUT (also recorded as sticky). */
int nnc_cuda_check_device_status(void);

void nnc_cuda_set_precision(int mode);
int nnc_cuda_get_precision(void);

/* ---- scratch memory ----------------------------------------------------------
 * Caller-owned workspace used by ops that need scratch (layout conversion for
 * NCHW conv calls, operand transposes, 3xTF32 operand splits). Passing NULL/0
 * returns to on-demand growth. */
int nnc_cuda_set_workspace(void* device_ptr, size_t bytes);
size_t nnc_cuda_get_workspace_capacity(void);

/* ---- prepacking of constant conv weights ------------------------------------
 * Re-lays a constant OIHW conv weight into the tensor-core layout (O, KH, KW,
 * I padded, TF32 hi/lo planes) at dst (device, bytes from
 * nnc_cuda_prepacked_conv_weight_bytes), then points w->data at dst and tags
 * w->dtype with NNC_CUDA_TAG_PACKED_CONV. Enqueued on the current stream. */
size_t nnc_cuda_prepacked_conv_weight_bytes(const Tensor* w);
int nnc_cuda_prepack_conv_weight(Tensor* w, void* dst, size_t dst_bytes);

/* ---- convolution that allocates nothing ---------------------------------------
 * No counterpart in the reference. nnc_conv (nnc_ops.h) with the same
 * arguments and results, for callers that must not allocate device memory
 * while they run. Its scratch (the NHWC copy of an NCHW input and the packed
 * weights; each twice in 3xTF32 mode) lives in a file-scope 16 MiB device
 * array, held by every GPU that loads the library until the process exits,
 * instead of the workspace that the other entry points grow with
 * cudaMallocAsync. It calls no cudaMalloc, cudaFree or other allocating
 * routine; a call whose scratch would exceed 16 MiB is rejected with
 * NNC_CUDA_ERR_INVALID before any work is queued.
 *   - Call nnc_cuda_init() on the device first (it creates the device's error
 *     word, which allocates); otherwise the call fails with
 *     NNC_CUDA_ERR_INVALID.
 *   - The first call on each device does the set-up: it resolves the array's
 *     device address (cudaGetSymbolAddress) with that device current. Make
 *     that first call before any stream capture.
 *   - All calls on a device share the array, which keeps the previous call's
 *     contents (nothing in it needs to start at zero: a call writes every
 *     scratch byte it reads before reading it). Calls that overlap on the GPU
 *     (other streams or threads on the same device) race on it. */
void nnc_conv_static_scratch(Tensor* input, Tensor* weight, Tensor* bias, Tensor* output,
                             int kernel_h, int kernel_w, int stride_h, int stride_w,
                             int pad_h, int pad_w);

/* ---- failure injection (tests of the error paths; no reference counterpart) --
 * nnc_cuda_inject_alloc_failures(n): the library's next n device allocations
 * (workspace growth; process-wide) fail as if the device were out of
 * memory: the op reports NNC_CUDA_ERR_NOMEM and queues nothing. 0 clears it.
 * nnc_cuda_selftest_bounded_wait(limit_us): queues one kernel whose thread
 * waits on an mbarrier that nothing completes, through the bounded wait the
 * tensor-core pipelines use, given up after limit_us microseconds (1 ..
 * 2000000): the kernel then records NNC_CUDA_ERR_DEVICE_TIMEOUT in the
 * device error word and returns, so nnc_cuda_check_device_status reports it
 * and the context stays usable. Neither faults nor hangs the GPU. */
void nnc_cuda_inject_alloc_failures(int count);
int nnc_cuda_selftest_bounded_wait(int limit_us);

/* ---- layout conversion at model boundaries (logical shapes are NCHW) ---- */
void nnc_cuda_nchw_to_nhwc(Tensor* input, Tensor* output);
void nnc_cuda_nhwc_to_nchw(Tensor* input, Tensor* output);

/* ---- plumbing for callers without their own CUDA runtime binding --------
 * Stream-ordered copy on the current stream; kind: 1 host->device,
 * 2 device->host, 3 device->device (cudaMemcpyKind values). */
int nnc_cuda_memcpy_async(void* dst, const void* src, size_t bytes, int kind);
/* Number of kernels this thread has launched through the library. */
long long nnc_cuda_launch_count(void);

/* ---- CUDA graphs (no reference counterpart: the x86 runtime has no launch
 * cost to hide) ----------------------------------------------------------------
 * nnc_cuda_graph_begin starts capturing this thread's current stream (a
 * stream set with nnc_cuda_set_stream); the library calls that follow are
 * recorded, not run, until nnc_cuda_graph_end, which returns a replayable
 * graph (NULL on failure: a call inside the capture failed, or the capture
 * was invalidated). Run the same calls once uncaptured first: the workspace
 * cannot grow during a capture. nnc_cuda_graph_launch replays the graph on
 * the current stream (its tensors' addresses are fixed at capture) and adds
 * its kernels to nnc_cuda_launch_count. A graph captured while tracing is on
 * holds two event-record nodes around each captured call; every replay made
 * while tracing is on logs those calls' device times in the trace below (one
 * record per call per replay), so operator times come from the replayed
 * graph itself. */
int nnc_cuda_graph_begin(void);
void* nnc_cuda_graph_end(void);
int nnc_cuda_graph_launch(void* graph);
long long nnc_cuda_graph_kernels(const void* graph);
void nnc_cuda_graph_destroy(void* graph);

/* ---- observability ------------------------------------------------------------
 * When enabled (or NNC_CUDA_TRACE=1 in the environment), every operator call
 * records CUDA events around its launches and the bytes of the tensors it
 * reads and writes. nnc_cuda_trace_dump prints the log to stdout in the line
 * format of nnc-py's costmodel runtime (runtime/x86/costmodel.c:253-357),
 *   [costmodel] #k op=<name> cu=<device> start=<t0> end=<t1> read=0
 *               compute=<t1 - t0> write=0 in=<bytes>B out=<bytes>B
 * one per call in issue order (k from 1), then
 *   [costmodel] summary ops=<n> total_cycles=<last end> shared_ready=<same>
 *   [costmodel] summary cu=<device> ready=<last end on that device>
 * with times in nanoseconds of device time since the first call's start
 * (where the costmodel prints simulated cycles; a kernel overlaps its reads
 * and writes with its arithmetic, so the whole duration is compute). It
 * returns the number of calls and clears the log. Synchronises the current
 * stream. */
void nnc_cuda_trace_enable(int on);
int nnc_cuda_trace_dump(void);
/* Programmatic access to the same log: nnc_cuda_trace_count synchronises
 * the current stream and returns the number of recorded calls; entry i has
 * an operator name and a device duration in microseconds. */
int nnc_cuda_trace_count(void);
const char* nnc_cuda_trace_name(int i);
float nnc_cuda_trace_us(int i);
void nnc_cuda_trace_clear(void);

#ifdef __cplusplus
}
#endif

#endif /* NNC_CUDA_H */
