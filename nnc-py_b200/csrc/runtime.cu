// Execution context of libnnc_cuda.so: per-thread device/stream/precision and
// sticky status, per-device error word, scratch memory, per-op tracing.
#include <stdarg.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>
#include <vector>

#include "common.cuh"
#include "tc.cuh"

namespace nnc {

namespace {
constexpr int kMaxDevices = 64;

struct DeviceState {
  bool ready = false;
  int* error_word = nullptr;  // device int, 0 = ok
  int sms = 148;
};
DeviceState g_dev[kMaxDevices];
std::mutex g_dev_mu;

struct Workspace {
  void* ptr[kMaxDevices] = {};
  size_t cap[kMaxDevices] = {};
  void* user_ptr[kMaxDevices] = {};
  size_t user_cap[kMaxDevices] = {};
};
thread_local Workspace t_ws;
// Failure injection: the next this-many device allocations of the library
// (workspace growth) fail as if the device were out of memory.
int g_fail_allocs = 0;
std::mutex g_fail_mu;

bool injected_alloc_failure() {
  std::lock_guard<std::mutex> lock(g_fail_mu);
  if (g_fail_allocs <= 0) return false;
  --g_fail_allocs;
  return true;
}

// One thread waits on a barrier that nothing completes, through the same
// bounded wait as the tensor-core pipelines, with a caller-chosen bound; the
// expired wait records the timeout in the device error word and the kernel
// returns.
__global__ void bounded_wait_selftest_kernel(int* err, uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, 1);
    tc::fence_barrier_init();
    tc::mbar_wait_for(&bar, 0, err, limit_ns);
  }
}

struct TraceRec {
  const char* name;
  cudaEvent_t start, stop;
  uint64_t in_bytes = 0, out_bytes = 0;  // tensor bytes the call reads / writes
  int device = 0;
};
thread_local std::vector<TraceRec> t_trace;
int g_trace_on = -1;  // -1: read NNC_CUDA_TRACE on first use
// Between nnc_cuda_graph_begin and nnc_cuda_graph_end: the calls of this
// thread are being captured (no workspace growth). With tracing on, each
// captured call is bracketed by two event-record nodes of the graph; the
// events are taken from a pool made before the capture started.
thread_local bool t_capturing = false;
thread_local long long t_capture_launches0 = 0;
thread_local std::vector<TraceRec> t_capture_ops;
thread_local std::vector<cudaEvent_t> t_capture_pool;
constexpr int kCaptureTraceEvents = 1024;

cudaEvent_t capture_event() {
  if (t_capture_pool.empty()) return nullptr;
  cudaEvent_t e = t_capture_pool.back();
  t_capture_pool.pop_back();
  return e;
}

bool trace_on() {
  if (g_trace_on < 0) {
    const char* e = getenv("NNC_CUDA_TRACE");
    g_trace_on = (e && e[0] == '1') ? 1 : 0;
  }
  return g_trace_on == 1;
}

DeviceState& dev_state(int dev) {
  DeviceState& s = g_dev[dev];
  if (!s.ready) {
    std::lock_guard<std::mutex> lock(g_dev_mu);
    if (!s.ready) {
      int prev = 0;
      cudaGetDevice(&prev);
      cudaSetDevice(dev);
      cudaDeviceGetAttribute(&s.sms, cudaDevAttrMultiProcessorCount, dev);
      if (cudaMalloc(&s.error_word, sizeof(int)) == cudaSuccess) {
        cudaMemset(s.error_word, 0, sizeof(int));
      } else {
        s.error_word = nullptr;
      }
      cudaSetDevice(prev);
      s.ready = true;
    }
  }
  return s;
}
}  // namespace

ThreadCtx& ctx() {
  thread_local ThreadCtx c;
  return c;
}

void fail(int code, const char* op, const char* fmt, ...) {
  ThreadCtx& c = ctx();
  char buf[400];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  if (c.status == NNC_CUDA_OK) {
    c.status = code;
    snprintf(c.message, sizeof(c.message), "%s: %s", op, buf);
  }
  fprintf(stderr, "%s: %s\n", op, buf);
  fflush(stderr);
}

bool check_cuda(cudaError_t err, const char* op, const char* what) {
  if (err == cudaSuccess) return true;
  fail(err == cudaErrorMemoryAllocation ? NNC_CUDA_ERR_NOMEM : NNC_CUDA_ERR_LAUNCH, op,
       "%s failed: %s", what, cudaGetErrorString(err));
  return false;
}

int* device_error_word() { return dev_state(ctx().device).error_word; }
bool device_ready() {
  const DeviceState& s = g_dev[ctx().device];
  return s.ready && s.error_word != nullptr;
}
int sm_count() { return dev_state(ctx().device).sms; }

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("NNC_CUDA_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

int grid_for(int64_t work_items, int threads, int max_ctas_per_sm) {
  int64_t want = cdiv(work_items, threads);
  int64_t cap = (int64_t)sm_count() * max_ctas_per_sm;
  if (want < 1) want = 1;
  return (int)(want < cap ? want : cap);
}

bool valid_tensor(const Tensor* t, const char* op, const char* name) {
  if (!t) {
    fail(NNC_CUDA_ERR_INVALID, op, "NULL tensor pointer (%s)", name);
    return false;
  }
  if (!t->shape && t->ndim > 0) {
    fail(NNC_CUDA_ERR_INVALID, op, "NULL shape pointer (%s)", name);
    return false;
  }
  if (t->ndim < 0 || t->ndim > 8) {
    fail(NNC_CUDA_ERR_INVALID, op, "ndim %d out of range (%s)", t->ndim, name);
    return false;
  }
  if (!t->data && numel(t) > 0) {
    fail(NNC_CUDA_ERR_INVALID, op, "NULL data pointer (%s)", name);
    return false;
  }
  return true;
}

void* workspace(size_t bytes, const char* op) {
  ThreadCtx& c = ctx();
  const int d = c.device;
  if (bytes == 0) bytes = 256;
  if (t_ws.user_ptr[d]) {
    if (bytes <= t_ws.user_cap[d]) return t_ws.user_ptr[d];
    fail(NNC_CUDA_ERR_NOMEM, op, "needs %zu bytes of workspace, caller supplied %zu", bytes,
         t_ws.user_cap[d]);
    return nullptr;
  }
  if (bytes <= t_ws.cap[d]) return t_ws.ptr[d];
  if (t_capturing) {
    // Memory allocated inside a graph lives only while the graph runs; the
    // workspace must already be large enough.
    fail(NNC_CUDA_ERR_INVALID, op,
         "needs %zu bytes of workspace while a graph is being captured (it holds %zu): run the "
         "same calls once before capturing them",
         bytes, t_ws.cap[d]);
    return nullptr;
  }
  // Grow stream-ordered: earlier work on this stream that still reads the
  // old buffer completes before the free takes effect.
  size_t want = bytes + bytes / 4;
  want = (want + (2u << 20) - 1) & ~size_t((2u << 20) - 1);
  if (t_ws.ptr[d]) {
    cudaFreeAsync(t_ws.ptr[d], c.stream);
    t_ws.ptr[d] = nullptr;
    t_ws.cap[d] = 0;
  }
  void* p = nullptr;
  if (injected_alloc_failure()) {
    fail(NNC_CUDA_ERR_NOMEM, op, "workspace allocation of %zu bytes failed (injected)", want);
    return nullptr;
  }
  if (!check_cuda(cudaMallocAsync(&p, want, c.stream), op, "workspace allocation")) return nullptr;
  t_ws.ptr[d] = p;
  t_ws.cap[d] = want;
  return p;
}

// Stream-K scratch of the paired conv kernel, per device for this thread:
// kStreamKCounterBytes of arrival counters (zeroed when allocated; every
// launch leaves them at zero) followed by the partial-accumulator slots.
struct StreamKScratch {
  void* ptr[kMaxDevices] = {};
  size_t cap[kMaxDevices] = {};
};
thread_local StreamKScratch t_sk;

bool streamk_scratch(int slots, size_t slot_bytes, unsigned** counters, float** parts) {
  ThreadCtx& c = ctx();
  const int d = c.device;
  if (slots <= 0 || (size_t)slots * sizeof(unsigned) > kStreamKCounterBytes) return false;
  const size_t bytes = kStreamKCounterBytes + (size_t)slots * slot_bytes;
  if (bytes > t_sk.cap[d]) {
    // Stream-K only saves time: it allocates nothing inside a capture or
    // beside a caller-supplied workspace, and a failed allocation just runs
    // the call without it.
    if (t_capturing || t_ws.user_ptr[d]) return false;
    if (t_sk.ptr[d]) {
      cudaFreeAsync(t_sk.ptr[d], c.stream);
      t_sk.ptr[d] = nullptr;
      t_sk.cap[d] = 0;
    }
    void* p = nullptr;
    if (cudaMallocAsync(&p, bytes, c.stream) != cudaSuccess) {
      cudaGetLastError();
      return false;
    }
    if (cudaMemsetAsync(p, 0, kStreamKCounterBytes, c.stream) != cudaSuccess) {
      cudaGetLastError();
      cudaFreeAsync(p, c.stream);
      return false;
    }
    t_sk.ptr[d] = p;
    t_sk.cap[d] = bytes;
  }
  *counters = (unsigned*)t_sk.ptr[d];
  *parts = (float*)((char*)t_sk.ptr[d] + kStreamKCounterBytes);
  return true;
}

// The innermost traced call of this thread (trace_io annotates it).
thread_local int t_scope_slot = -1;
thread_local bool t_scope_captured = false;

OpScope::OpScope(const char* name)
    : name_(name), slot_(-1), prev_slot_(t_scope_slot), prev_captured_(t_scope_captured) {
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < kMaxDevices) ctx().device = dev;
  t_scope_slot = -1;
  if (!trace_on()) return;
  if (t_capturing) {
    // Captured call: event-record nodes in the graph (re-bound to fresh
    // events at every traced replay by nnc_cuda_graph_launch).
    if (t_capture_pool.size() < 2) return;
    TraceRec r{name, capture_event(), capture_event()};
    r.device = ctx().device;
    cudaEventRecordWithFlags(r.start, ctx().stream, cudaEventRecordExternal);
    t_capture_ops.push_back(r);
    slot_ = (int)t_capture_ops.size() - 1;
    t_scope_slot = slot_;
    t_scope_captured = true;
    return;
  }
  TraceRec r{name, nullptr, nullptr};
  r.device = ctx().device;
  cudaEventCreate(&r.start);
  cudaEventCreate(&r.stop);
  cudaEventRecord(r.start, ctx().stream);
  t_trace.push_back(r);
  slot_ = (int)t_trace.size() - 1;
  t_scope_slot = slot_;
  t_scope_captured = false;
}

OpScope::~OpScope() {
  t_scope_slot = prev_slot_;
  t_scope_captured = prev_captured_;
  if (slot_ < 0) return;
  if (t_capturing) {
    if (slot_ < (int)t_capture_ops.size())
      cudaEventRecordWithFlags(t_capture_ops[slot_].stop, ctx().stream, cudaEventRecordExternal);
    return;
  }
  if (slot_ < (int)t_trace.size()) cudaEventRecord(t_trace[slot_].stop, ctx().stream);
}

uint64_t tensor_bytes(const Tensor* t) {
  if (!t) return 0;
  if (t->nbytes > 0) return (uint64_t)t->nbytes;
  if (t->ndim > 0 && !t->shape) return 0;
  return (uint64_t)numel(t) * elem_size(elem_type(t));
}

void trace_io(uint64_t in_bytes, uint64_t out_bytes) {
  if (t_scope_slot < 0) return;
  std::vector<TraceRec>& v = t_scope_captured ? t_capture_ops : t_trace;
  // The first annotation of a call wins: helpers it runs (a conv into a
  // temporary, a softmax after a contraction) do not overwrite it.
  if (t_scope_slot < (int)v.size() && v[t_scope_slot].in_bytes == 0 && v[t_scope_slot].out_bytes == 0) {
    v[t_scope_slot].in_bytes = in_bytes;
    v[t_scope_slot].out_bytes = out_bytes;
  }
}

}  // namespace nnc

using namespace nnc;

extern "C" {

int nnc_cuda_init(int device) {
  int count = 0;
  if (!check_cuda(cudaGetDeviceCount(&count), "nnc_cuda_init", "cudaGetDeviceCount")) return ctx().status;
  if (device < 0 || device >= count || device >= 64) {
    fail(NNC_CUDA_ERR_INVALID, "nnc_cuda_init", "device %d out of range (%d devices)", device, count);
    return NNC_CUDA_ERR_INVALID;
  }
  if (!check_cuda(cudaSetDevice(device), "nnc_cuda_init", "cudaSetDevice")) return ctx().status;
  ctx().device = device;
  DeviceState& s = dev_state(device);
  if (!s.error_word) {
    fail(NNC_CUDA_ERR_NOMEM, "nnc_cuda_init", "could not allocate the device error word");
    return NNC_CUDA_ERR_NOMEM;
  }
  return NNC_CUDA_OK;
}

int nnc_cuda_set_device(int device) { return nnc_cuda_init(device); }
int nnc_cuda_get_device(void) { return ctx().device; }
void nnc_cuda_set_stream(void* stream) { ctx().stream = (cudaStream_t)stream; }
void* nnc_cuda_get_stream(void) { return (void*)ctx().stream; }

int nnc_cuda_sync(void) {
  check_cuda(cudaStreamSynchronize(ctx().stream), "nnc_cuda_sync", "cudaStreamSynchronize");
  return ctx().status;
}

int nnc_cuda_get_last_error(void) { return ctx().status; }
const char* nnc_cuda_get_last_error_string(void) { return ctx().message; }
void nnc_cuda_clear_error(void) {
  ctx().status = NNC_CUDA_OK;
  ctx().message[0] = 0;
}

int nnc_cuda_check_device_status(void) {
  int* w = device_error_word();
  if (!w) return ctx().status;
  int h = 0;
  if (!check_cuda(cudaStreamSynchronize(ctx().stream), "nnc_cuda_check_device_status", "sync"))
    return ctx().status;
  if (!check_cuda(cudaMemcpy(&h, w, sizeof(int), cudaMemcpyDeviceToHost),
                  "nnc_cuda_check_device_status", "read error word"))
    return ctx().status;
  if (h != 0) {
    cudaMemset(w, 0, sizeof(int));
    // An expired wait may have left stream-K arrival counters non-zero.
    if (t_sk.ptr[ctx().device]) cudaMemset(t_sk.ptr[ctx().device], 0, kStreamKCounterBytes);
    fail(NNC_CUDA_ERR_DEVICE_TIMEOUT, "nnc_cuda_check_device_status",
         "a kernel's bounded wait expired (code %d)", h);
    return NNC_CUDA_ERR_DEVICE_TIMEOUT;
  }
  return NNC_CUDA_OK;
}

void nnc_cuda_set_precision(int mode) {
  ctx().precision = (mode == NNC_CUDA_PRECISION_3XTF32) ? NNC_CUDA_PRECISION_3XTF32
                                                         : NNC_CUDA_PRECISION_TF32;
}
int nnc_cuda_get_precision(void) { return ctx().precision; }

int nnc_cuda_set_workspace(void* device_ptr, size_t bytes) {
  const int d = ctx().device;
  t_ws.user_ptr[d] = bytes ? device_ptr : nullptr;
  t_ws.user_cap[d] = device_ptr ? bytes : 0;
  return NNC_CUDA_OK;
}

size_t nnc_cuda_get_workspace_capacity(void) {
  const int d = ctx().device;
  return t_ws.user_ptr[d] ? t_ws.user_cap[d] : t_ws.cap[d];
}

int nnc_cuda_memcpy_async(void* dst, const void* src, size_t bytes, int kind) {
  if (kind < 1 || kind > 3) {
    fail(NNC_CUDA_ERR_INVALID, "nnc_cuda_memcpy_async", "kind %d is not 1, 2 or 3", kind);
    return NNC_CUDA_ERR_INVALID;
  }
  if (!check_cuda(cudaMemcpyAsync(dst, src, bytes, (cudaMemcpyKind)kind, ctx().stream),
                  "nnc_cuda_memcpy_async", "cudaMemcpyAsync"))
    return ctx().status;
  return NNC_CUDA_OK;
}

long long nnc_cuda_launch_count(void) { return ctx().launches; }

void nnc_cuda_inject_alloc_failures(int count) {
  std::lock_guard<std::mutex> lock(g_fail_mu);
  g_fail_allocs = count > 0 ? count : 0;
}

int nnc_cuda_selftest_bounded_wait(int limit_us) {
  const char* op = "nnc_cuda_selftest_bounded_wait";
  OpScope scope(op);
  if (limit_us < 1 || limit_us > 2000000) {
    fail(NNC_CUDA_ERR_INVALID, op, "limit %d us outside [1, 2000000]", limit_us);
    return NNC_CUDA_ERR_INVALID;
  }
  int* err = device_error_word();
  if (!err) {
    fail(NNC_CUDA_ERR_NOMEM, op, "no device error word");
    return NNC_CUDA_ERR_NOMEM;
  }
  bounded_wait_selftest_kernel<<<1, 32, 0, ctx().stream>>>(err, (uint64_t)limit_us * 1000ull);
  if (!check_launch(op)) return ctx().status;
  return NNC_CUDA_OK;
}

// ---- CUDA graphs ---------------------------------------------------------
// A traced call inside a captured graph: its two event-record nodes and the
// events the graph owns for them (bound whenever a replay is not traced).
struct GraphOp {
  const char* name;
  cudaGraphNode_t start_node, stop_node;
  cudaEvent_t own_start, own_stop;
  uint64_t in_bytes, out_bytes;
  int device;
};

struct NncGraph {
  cudaGraph_t graph;  // kept while the exec graph lives when it holds trace nodes
  cudaGraphExec_t exec;
  long long kernels;  // library kernels in one replay
  std::vector<GraphOp> ops;
  bool own_bound;  // the exec graph's trace nodes record into the own events
};

namespace {
// This thread's live graphs that hold trace nodes: nnc_cuda_trace_clear
// re-binds them to their own events before it destroys the logged ones.
thread_local std::vector<NncGraph*> t_traced_graphs;

void release_capture_trace() {
  for (auto& r : t_capture_ops) {
    cudaEventDestroy(r.start);
    cudaEventDestroy(r.stop);
  }
  t_capture_ops.clear();
  for (cudaEvent_t e : t_capture_pool) cudaEventDestroy(e);
  t_capture_pool.clear();
}

// Binds a traced graph's event-record nodes to fresh events and logs them as
// one trace record per captured call (this replay's device times).
bool bind_trace_events(NncGraph* g, const char* op) {
  for (const GraphOp& o : g->ops) {
    TraceRec r{o.name, nullptr, nullptr, o.in_bytes, o.out_bytes, o.device};
    if (!check_cuda(cudaEventCreate(&r.start), op, "cudaEventCreate") ||
        !check_cuda(cudaEventCreate(&r.stop), op, "cudaEventCreate"))
      return false;
    if (!check_cuda(cudaGraphExecEventRecordNodeSetEvent(g->exec, o.start_node, r.start), op,
                    "cudaGraphExecEventRecordNodeSetEvent") ||
        !check_cuda(cudaGraphExecEventRecordNodeSetEvent(g->exec, o.stop_node, r.stop), op,
                    "cudaGraphExecEventRecordNodeSetEvent"))
      return false;
    t_trace.push_back(r);
  }
  g->own_bound = false;
  return true;
}

bool bind_own_events(NncGraph* g, const char* op) {
  for (const GraphOp& o : g->ops) {
    if (!check_cuda(cudaGraphExecEventRecordNodeSetEvent(g->exec, o.start_node, o.own_start), op,
                    "cudaGraphExecEventRecordNodeSetEvent") ||
        !check_cuda(cudaGraphExecEventRecordNodeSetEvent(g->exec, o.stop_node, o.own_stop), op,
                    "cudaGraphExecEventRecordNodeSetEvent"))
      return false;
  }
  g->own_bound = true;
  return true;
}

void destroy_graph(NncGraph* g) {
  for (size_t i = 0; i < t_traced_graphs.size(); ++i) {
    if (t_traced_graphs[i] == g) {
      t_traced_graphs.erase(t_traced_graphs.begin() + i);
      break;
    }
  }
  if (g->exec) cudaGraphExecDestroy(g->exec);
  if (g->graph) cudaGraphDestroy(g->graph);
  for (auto& o : g->ops) {
    cudaEventDestroy(o.own_start);
    cudaEventDestroy(o.own_stop);
  }
  delete g;
}
}  // namespace

int nnc_cuda_graph_begin(void) {
  const char* op = "nnc_cuda_graph_begin";
  if (t_capturing) {
    fail(NNC_CUDA_ERR_INVALID, op, "a capture is already open on this thread");
    return NNC_CUDA_ERR_INVALID;
  }
  if (ctx().stream == nullptr) {
    fail(NNC_CUDA_ERR_INVALID, op, "capture needs a created stream (nnc_cuda_set_stream), not the "
                                   "legacy default stream");
    return NNC_CUDA_ERR_INVALID;
  }
  release_capture_trace();
  if (trace_on()) {
    // Events for the captured calls' trace nodes, made before the capture.
    for (int i = 0; i < kCaptureTraceEvents; ++i) {
      cudaEvent_t e = nullptr;
      if (!check_cuda(cudaEventCreate(&e), op, "cudaEventCreate")) {
        release_capture_trace();
        return ctx().status;
      }
      t_capture_pool.push_back(e);
    }
  }
  if (!check_cuda(cudaStreamBeginCapture(ctx().stream, cudaStreamCaptureModeThreadLocal), op,
                  "cudaStreamBeginCapture")) {
    release_capture_trace();
    return ctx().status;
  }
  t_capturing = true;
  t_capture_launches0 = ctx().launches;
  return NNC_CUDA_OK;
}

void* nnc_cuda_graph_end(void) {
  const char* op = "nnc_cuda_graph_end";
  if (!t_capturing) {
    fail(NNC_CUDA_ERR_INVALID, op, "no capture is open on this thread");
    return nullptr;
  }
  t_capturing = false;
  cudaGraph_t graph = nullptr;
  if (!check_cuda(cudaStreamEndCapture(ctx().stream, &graph), op, "cudaStreamEndCapture")) {
    release_capture_trace();
    return nullptr;
  }
  const long long kernels = ctx().launches - t_capture_launches0;
  ctx().launches = t_capture_launches0;  // captured, not launched
  if (ctx().status != NNC_CUDA_OK) {  // a call inside the capture failed
    cudaGraphDestroy(graph);
    release_capture_trace();
    return nullptr;
  }
  NncGraph* g = new NncGraph{nullptr, nullptr, kernels, {}, true};
  if (!t_capture_ops.empty()) {
    // Find each traced call's two event-record nodes by their events.
    size_t n = 0;
    cudaGraphGetNodes(graph, nullptr, &n);
    std::vector<cudaGraphNode_t> nodes(n);
    if (n) cudaGraphGetNodes(graph, nodes.data(), &n);
    for (const TraceRec& r : t_capture_ops)
      g->ops.push_back(GraphOp{r.name, nullptr, nullptr, r.start, r.stop, r.in_bytes, r.out_bytes, r.device});
    for (cudaGraphNode_t node : nodes) {
      cudaGraphNodeType type;
      if (cudaGraphNodeGetType(node, &type) != cudaSuccess || type != cudaGraphNodeTypeEventRecord)
        continue;
      cudaEvent_t e = nullptr;
      if (cudaGraphEventRecordNodeGetEvent(node, &e) != cudaSuccess) continue;
      for (GraphOp& o : g->ops) {
        if (o.own_start == e) o.start_node = node;
        if (o.own_stop == e) o.stop_node = node;
      }
    }
    t_capture_ops.clear();  // the events now belong to the graph
    bool found = true;
    for (const GraphOp& o : g->ops) found = found && o.start_node && o.stop_node;
    if (!found) {
      fail(NNC_CUDA_ERR_LAUNCH, op, "trace nodes of the captured calls not found in the graph");
      cudaGraphDestroy(graph);
      destroy_graph(g);
      release_capture_trace();
      return nullptr;
    }
  }
  release_capture_trace();
  const bool ok = check_cuda(cudaGraphInstantiate(&g->exec, graph, 0), op, "cudaGraphInstantiate");
  if (g->ops.empty()) {
    cudaGraphDestroy(graph);
  } else {
    g->graph = graph;  // node handles stay valid while the graph exists
  }
  if (!ok) {
    destroy_graph(g);
    return nullptr;
  }
  if (!g->ops.empty()) t_traced_graphs.push_back(g);
  return g;
}

int nnc_cuda_graph_launch(void* graph) {
  const char* op = "nnc_cuda_graph_launch";
  if (!graph) {
    fail(NNC_CUDA_ERR_INVALID, op, "NULL graph");
    return NNC_CUDA_ERR_INVALID;
  }
  NncGraph* g = static_cast<NncGraph*>(graph);
  if (!g->ops.empty()) {
    // A graph captured with tracing: a traced replay logs its calls' device
    // times; an untraced one records into the graph's own events. Rebinding
    // affects this and later replays only, never one already queued.
    if (trace_on()) {
      if (!bind_trace_events(g, op)) return ctx().status;
    } else if (!g->own_bound) {
      if (!bind_own_events(g, op)) return ctx().status;
    }
  }
  if (!check_cuda(cudaGraphLaunch(g->exec, ctx().stream), op, "cudaGraphLaunch")) return ctx().status;
  ctx().launches += g->kernels;
  return NNC_CUDA_OK;
}

long long nnc_cuda_graph_kernels(const void* graph) {
  return graph ? static_cast<const NncGraph*>(graph)->kernels : 0;
}

void nnc_cuda_graph_destroy(void* graph) {
  if (!graph) return;
  destroy_graph(static_cast<NncGraph*>(graph));
}

int nnc_cuda_trace_count(void) {
  cudaStreamSynchronize(ctx().stream);
  return (int)t_trace.size();
}

const char* nnc_cuda_trace_name(int i) {
  return (i >= 0 && i < (int)t_trace.size()) ? t_trace[i].name : "";
}

float nnc_cuda_trace_us(int i) {
  if (i < 0 || i >= (int)t_trace.size()) return -1.f;
  float ms = 0.f;
  if (cudaEventElapsedTime(&ms, t_trace[i].start, t_trace[i].stop) != cudaSuccess) return -1.f;
  return ms * 1e3f;
}

void nnc_cuda_trace_clear(void) {
  // The logged events may still be bound to a traced graph's nodes (its last
  // traced replay): bind the graph's own events first, then wait for the
  // replays that record into the logged ones.
  for (NncGraph* g : t_traced_graphs)
    if (!g->own_bound) bind_own_events(g, "nnc_cuda_trace_clear");
  cudaStreamSynchronize(ctx().stream);
  for (auto& r : t_trace) {
    cudaEventDestroy(r.start);
    cudaEventDestroy(r.stop);
  }
  t_trace.clear();
}

void nnc_cuda_trace_enable(int on) { g_trace_on = on ? 1 : 0; }

int nnc_cuda_trace_dump(void) {
  cudaStreamSynchronize(ctx().stream);
  if (t_trace.empty()) return 0;
  const int n = (int)t_trace.size();
  // The costmodel runtime's line format (one line per call, then a summary;
  // nnc-py runtime/x86/costmodel.c): times are device nanoseconds since the
  // first traced call's start instead of simulated cycles, `cu` is the
  // device, and the whole duration counts as compute (a kernel overlaps its
  // reads and writes with its arithmetic).
  cudaEvent_t t0 = t_trace[0].start;
  uint64_t total = 0;
  std::vector<std::pair<int, uint64_t>> ready;  // (device, last end)
  for (int i = 0; i < n; ++i) {
    float s = 0.f, e = 0.f;
    cudaEventElapsedTime(&s, t0, t_trace[i].start);
    cudaEventElapsedTime(&e, t0, t_trace[i].stop);
    const uint64_t start = (uint64_t)(s * 1e6 + 0.5), end = (uint64_t)(e * 1e6 + 0.5);
    const TraceRec& r = t_trace[i];
    printf("[costmodel] #%d op=%s cu=%d start=%llu end=%llu read=0 compute=%llu write=0 in=%lluB "
           "out=%lluB\n",
           i + 1, r.name, r.device, (unsigned long long)start, (unsigned long long)end,
           (unsigned long long)(end > start ? end - start : 0), (unsigned long long)r.in_bytes,
           (unsigned long long)r.out_bytes);
    if (end > total) total = end;
    bool found = false;
    for (auto& d : ready)
      if (d.first == r.device) {
        if (end > d.second) d.second = end;
        found = true;
      }
    if (!found) ready.push_back({r.device, end});
  }
  printf("[costmodel] summary ops=%d total_cycles=%llu shared_ready=%llu\n", n,
         (unsigned long long)total, (unsigned long long)total);
  for (auto& d : ready)
    printf("[costmodel] summary cu=%d ready=%llu\n", d.first, (unsigned long long)d.second);
  fflush(stdout);
  nnc_cuda_trace_clear();
  return n;
}

}  // extern "C"
