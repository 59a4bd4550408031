// The mcpu device runtime C-ABI (include/openreg.h) over the CUDA runtime.
//
// Reference: third_party/openreg/csrc/{memory.cpp,stream.cpp,device.cpp} of
// kzwrime/torch_mcpu, where the "device" is host memory served by worker
// threads.  Here every call maps onto its CUDA counterpart; the reference's
// host-side timeouts (stream.cpp:229-240, 321-383) are kept by polling.
#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <thread>
#include <utility>

#include "common.cuh"

namespace mcpu {

static thread_local char g_last_error[512] = {0};

void set_last_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

orError_t from_cuda(cudaError_t st, const char* what) {
  if (st == cudaSuccess) return orSuccess;
  if (st == cudaErrorNotReady) return orErrorNotReady;
  set_last_error("%s: %s (%s)", what, cudaGetErrorString(st), cudaGetErrorName(st));
  if (st == cudaErrorInvalidValue) return orErrorInvalidValue;
  return orErrorUnknown;
}

// TORCH_MCPU_STREAM_SYNC_TIMEOUT_MS: 0 or unset = wait without a deadline.
static long sync_timeout_ms() {
  const char* v = std::getenv("TORCH_MCPU_STREAM_SYNC_TIMEOUT_MS");
  if (!v || !*v) return 0;
  long ms = std::strtol(v, nullptr, 10);
  return ms > 0 ? ms : 0;
}

template <typename Query>
static orError_t poll_until(Query q, const char* what) {
  long limit = sync_timeout_ms();
  auto start = std::chrono::steady_clock::now();
  for (unsigned spins = 0;; ++spins) {
    cudaError_t st = q();
    if (st == cudaSuccess) return orSuccess;
    if (st != cudaErrorNotReady) return from_cuda(st, what);
    if (limit > 0) {
      auto el = std::chrono::duration_cast<std::chrono::milliseconds>(
                    std::chrono::steady_clock::now() - start)
                    .count();
      if (el >= limit) {
        set_last_error("%s: timed out after %ld ms (TORCH_MCPU_STREAM_SYNC_TIMEOUT_MS)", what,
                       (long)el);
        return orErrorTimeout;
      }
    }
    if (spins > 64) std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

cudaError_t ensure_dynamic_smem(const void* kernel, int bytes) {
  // cudaFuncSetAttribute acts on the current device's context only, so the
  // raised limit is recorded per (kernel, device); the map is shared by all
  // host threads.
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> raised;
  int dev = 0;
  cudaError_t st = cudaGetDevice(&dev);
  if (st != cudaSuccess) return st;
  std::lock_guard<std::mutex> lock(mu);
  int& have = raised[std::make_pair(kernel, dev)];
  if (have >= bytes) return cudaSuccess;
  st = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (st == cudaSuccess) have = bytes;
  return st;
}

void* driver_entry(const char* name) {
  void* ptr = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &ptr, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess)
    return nullptr;
  return ptr;
}

}  // namespace mcpu

using namespace mcpu;

extern "C" {

const char* mcpuGetLastErrorString(void) { return g_last_error; }

// ------------------------------------------------------------------ graphs
orError_t mcpu_graph_capture_begin(orStream_t stream) {
  MCPU_ARG_CHECK(stream != nullptr, "graph capture: a created stream is needed");
  return from_cuda(cudaStreamBeginCapture(as_cuda(stream), cudaStreamCaptureModeThreadLocal),
                   "cudaStreamBeginCapture");
}

orError_t mcpu_graph_capture_end(orStream_t stream, void** graph_exec) {
  MCPU_ARG_CHECK(stream != nullptr && graph_exec != nullptr, "graph capture end: NULL argument");
  cudaGraph_t graph = nullptr;
  MCPU_CUDA_TRY(cudaStreamEndCapture(as_cuda(stream), &graph), "cudaStreamEndCapture");
  cudaGraphExec_t exec = nullptr;
  const cudaError_t e = cudaGraphInstantiate(&exec, graph, 0);
  cudaGraphDestroy(graph);
  if (e != cudaSuccess) return from_cuda(e, "cudaGraphInstantiate");
  *graph_exec = exec;
  return orSuccess;
}

orError_t mcpu_graph_launch(void* graph_exec, orStream_t stream) {
  MCPU_ARG_CHECK(graph_exec != nullptr, "graph launch: NULL graph");
  return from_cuda(cudaGraphLaunch(static_cast<cudaGraphExec_t>(graph_exec), as_cuda(stream)),
                   "cudaGraphLaunch");
}

orError_t mcpu_graph_destroy(void* graph_exec) {
  if (!graph_exec) return orSuccess;
  return from_cuda(cudaGraphExecDestroy(static_cast<cudaGraphExec_t>(graph_exec)), "cudaGraphExecDestroy");
}

orError_t mcpu_device_error(int* flag, int reset) {
  MCPU_ARG_CHECK(flag != nullptr, "mcpu_device_error: flag is NULL");
  int a = 0, b = 0, c = 0;
  orError_t e = gemm::read_error(&a, reset != 0);
  if (e != orSuccess) return e;
  e = router::read_error(&b, reset != 0);
  if (e != orSuccess) return e;
  e = bw::read_error(&c, reset != 0);
  if (e != orSuccess) return e;
  int d = 0, m = 0;
  e = aten_read_error(&d, reset != 0);
  if (e != orSuccess) return e;
  e = moe_read_error(&m, reset != 0);
  if (e != orSuccess) return e;
  int sp = 0;
  e = sampler_read_error(&sp, reset != 0);
  if (e != orSuccess) return e;
  *flag = a | b | c | d | m | sp;
  return orSuccess;
}

// ------------------------------------------------------------------ memory
orError_t orMalloc(void** devPtr, size_t size) {
  MCPU_ARG_CHECK(devPtr != nullptr, "orMalloc: devPtr is NULL");
  return from_cuda(cudaMalloc(devPtr, size), "orMalloc");
}

orError_t orFree(void* devPtr) {
  if (!devPtr) return orSuccess;
  return from_cuda(cudaFree(devPtr), "orFree");
}

orError_t orMallocHost(void** hostPtr, size_t size) {
  MCPU_ARG_CHECK(hostPtr != nullptr, "orMallocHost: hostPtr is NULL");
  return from_cuda(cudaMallocHost(hostPtr, size), "orMallocHost");
}

orError_t orFreeHost(void* hostPtr) {
  if (!hostPtr) return orSuccess;
  return from_cuda(cudaFreeHost(hostPtr), "orFreeHost");
}

static bool map_kind(orMemcpyKind k, cudaMemcpyKind* out) {
  switch (k) {
    case orMemcpyHostToHost: *out = cudaMemcpyHostToHost; return true;
    case orMemcpyHostToDevice: *out = cudaMemcpyHostToDevice; return true;
    case orMemcpyDeviceToHost: *out = cudaMemcpyDeviceToHost; return true;
    case orMemcpyDeviceToDevice: *out = cudaMemcpyDeviceToDevice; return true;
  }
  return false;
}

// The reference checks that each pointer lives where `kind` says
// (third_party/openreg/csrc/memory.cpp:104-154); CUDA reports such
// mismatches itself through cudaErrorInvalidValue.
orError_t orMemcpy(void* dst, const void* src, size_t count, orMemcpyKind kind) {
  cudaMemcpyKind ck;
  MCPU_ARG_CHECK(map_kind(kind, &ck), "orMemcpy: bad kind %d", (int)kind);
  if (count == 0) return orSuccess;
  MCPU_ARG_CHECK(dst && src, "orMemcpy: NULL pointer");
  return from_cuda(cudaMemcpy(dst, src, count, ck), "orMemcpy");
}

orError_t orMemcpyAsync(void* dst, const void* src, size_t count, orMemcpyKind kind,
                        orStream_t stream) {
  cudaMemcpyKind ck;
  MCPU_ARG_CHECK(map_kind(kind, &ck), "orMemcpyAsync: bad kind %d", (int)kind);
  if (count == 0) return orSuccess;
  MCPU_ARG_CHECK(dst && src, "orMemcpyAsync: NULL pointer");
  return from_cuda(cudaMemcpyAsync(dst, src, count, ck, as_cuda(stream)), "orMemcpyAsync");
}

orError_t orPointerGetAttributes(orPointerAttributes* attributes, const void* ptr) {
  MCPU_ARG_CHECK(attributes != nullptr, "orPointerGetAttributes: attributes is NULL");
  cudaPointerAttributes a;
  cudaError_t st = cudaPointerGetAttributes(&a, ptr);
  if (st != cudaSuccess) {
    cudaGetLastError();
    attributes->type = orMemoryTypeUnmanaged;
    attributes->device = -1;
    attributes->pointer = const_cast<void*>(ptr);
    return orSuccess;
  }
  switch (a.type) {
    case cudaMemoryTypeDevice:
    case cudaMemoryTypeManaged:
      attributes->type = orMemoryTypeDevice;
      break;
    case cudaMemoryTypeHost:
      attributes->type = orMemoryTypeHost;
      break;
    default:
      attributes->type = orMemoryTypeUnmanaged;
  }
  attributes->device = a.device;
  attributes->pointer = const_cast<void*>(ptr);
  return orSuccess;
}

orError_t orMemoryUnprotect(void*) { return orSuccess; }
orError_t orMemoryProtect(void*) { return orSuccess; }

// ------------------------------------------------------------------ device
orError_t orGetDeviceCount(int* count) {
  MCPU_ARG_CHECK(count != nullptr, "orGetDeviceCount: count is NULL");
  cudaError_t st = cudaGetDeviceCount(count);
  if (st != cudaSuccess) {
    *count = 0;
    return from_cuda(st, "orGetDeviceCount");
  }
  return orSuccess;
}

orError_t orSetDevice(int device) { return from_cuda(cudaSetDevice(device), "orSetDevice"); }

orError_t orGetDevice(int* device) {
  MCPU_ARG_CHECK(device != nullptr, "orGetDevice: device is NULL");
  return from_cuda(cudaGetDevice(device), "orGetDevice");
}

orError_t orDeviceGetStreamPriorityRange(int* leastPriority, int* greatestPriority) {
  // reference convention (third_party/openreg/csrc/stream.cpp:668-678)
  if (leastPriority) *leastPriority = 1;
  if (greatestPriority) *greatestPriority = 0;
  return orSuccess;
}

orError_t orDeviceSynchronize(void) {
  return from_cuda(cudaDeviceSynchronize(), "orDeviceSynchronize");
}

// ------------------------------------------------------------------ streams
static int to_cuda_priority(int p) {
  int least = 0, greatest = 0;
  cudaDeviceGetStreamPriorityRange(&least, &greatest);
  return p <= 0 ? greatest : least;
}

orError_t orStreamCreateWithPriority(orStream_t* stream, unsigned int /*flags*/, int priority) {
  MCPU_ARG_CHECK(stream != nullptr, "orStreamCreateWithPriority: stream is NULL");
  cudaStream_t s = nullptr;
  MCPU_CUDA_TRY(cudaStreamCreateWithPriority(&s, cudaStreamNonBlocking, to_cuda_priority(priority)),
                "orStreamCreateWithPriority");
  *stream = reinterpret_cast<orStream_t>(s);
  return orSuccess;
}

orError_t orStreamCreate(orStream_t* stream) {
  return orStreamCreateWithPriority(stream, orStreamDefault, 1);
}

orError_t orStreamGetPriority(orStream_t stream, int* priority) {
  MCPU_ARG_CHECK(priority != nullptr, "orStreamGetPriority: priority is NULL");
  int p = 0, least = 0, greatest = 0;
  MCPU_CUDA_TRY(cudaStreamGetPriority(as_cuda(stream), &p), "orStreamGetPriority");
  cudaDeviceGetStreamPriorityRange(&least, &greatest);
  *priority = (p == greatest && greatest != least) ? 0 : 1;
  return orSuccess;
}

// Like the reference (stream.cpp:604-628) the stream is drained first; a
// stream that does not drain within the sync timeout is reported, not freed.
orError_t orStreamDestroy(orStream_t stream) {
  MCPU_ARG_CHECK(stream != nullptr, "orStreamDestroy: NULL stream");
  orError_t st = orStreamSynchronize(stream);
  if (st != orSuccess) return st;
  return from_cuda(cudaStreamDestroy(as_cuda(stream)), "orStreamDestroy");
}

orError_t orStreamQuery(orStream_t stream) {
  return from_cuda(cudaStreamQuery(as_cuda(stream)), "orStreamQuery");
}

orError_t orStreamSynchronize(orStream_t stream) {
  if (sync_timeout_ms() == 0)
    return from_cuda(cudaStreamSynchronize(as_cuda(stream)), "orStreamSynchronize");
  cudaStream_t s = as_cuda(stream);
  return poll_until([s] { return cudaStreamQuery(s); }, "orStreamSynchronize");
}

orError_t orStreamWaitEvent(orStream_t stream, orEvent_t event, unsigned int flags) {
  MCPU_ARG_CHECK(event != nullptr, "orStreamWaitEvent: NULL event");
  return from_cuda(cudaStreamWaitEvent(as_cuda(stream), reinterpret_cast<cudaEvent_t>(event), flags),
                   "orStreamWaitEvent");
}

// ------------------------------------------------------------------ events
orError_t orEventCreateWithFlags(orEvent_t* event, unsigned int flags) {
  MCPU_ARG_CHECK(event != nullptr, "orEventCreateWithFlags: event is NULL");
  unsigned cf = (flags & orEventEnableTiming) ? cudaEventDefault : cudaEventDisableTiming;
  cudaEvent_t e = nullptr;
  MCPU_CUDA_TRY(cudaEventCreateWithFlags(&e, cf), "orEventCreateWithFlags");
  *event = reinterpret_cast<orEvent_t>(e);
  return orSuccess;
}

orError_t orEventCreate(orEvent_t* event) {
  return orEventCreateWithFlags(event, orEventDisableTiming);
}

orError_t orEventDestroy(orEvent_t event) {
  MCPU_ARG_CHECK(event != nullptr, "orEventDestroy: NULL event");
  return from_cuda(cudaEventDestroy(reinterpret_cast<cudaEvent_t>(event)), "orEventDestroy");
}

orError_t orEventRecord(orEvent_t event, orStream_t stream) {
  MCPU_ARG_CHECK(event != nullptr, "orEventRecord: NULL event");
  return from_cuda(cudaEventRecord(reinterpret_cast<cudaEvent_t>(event), as_cuda(stream)),
                   "orEventRecord");
}

orError_t orEventSynchronize(orEvent_t event) {
  MCPU_ARG_CHECK(event != nullptr, "orEventSynchronize: NULL event");
  cudaEvent_t e = reinterpret_cast<cudaEvent_t>(event);
  if (sync_timeout_ms() == 0) return from_cuda(cudaEventSynchronize(e), "orEventSynchronize");
  return poll_until([e] { return cudaEventQuery(e); }, "orEventSynchronize");
}

orError_t orEventQuery(orEvent_t event) {
  MCPU_ARG_CHECK(event != nullptr, "orEventQuery: NULL event");
  return from_cuda(cudaEventQuery(reinterpret_cast<cudaEvent_t>(event)), "orEventQuery");
}

orError_t orEventElapsedTime(float* ms, orEvent_t start, orEvent_t end) {
  MCPU_ARG_CHECK(ms && start && end, "orEventElapsedTime: NULL argument");
  return from_cuda(cudaEventElapsedTime(ms, reinterpret_cast<cudaEvent_t>(start),
                                        reinterpret_cast<cudaEvent_t>(end)),
                   "orEventElapsedTime");
}

}  // extern "C"
