// The "mcpu" PrivateUse1 device of PyTorch, backed by B200 memory.
//
// Mirrors the reference's backend core (kzwrime/torch_mcpu csrc/runtime and
// csrc/aten) as a host layer over the C-ABI of include/openreg.h and
// include/mcpu_ops.h; nothing here touches CUDA directly:
//   allocator   csrc/runtime/DeviceCachingAllocator.cpp -> stream-ordered
//               orMallocAsync/orFreeAsync; record_stream defers the free
//               behind events recorded on every stream that used the block
//   guard       csrc/runtime/OpenRegGuard.h:46-320 (device, streams, events)
//   streams     csrc/runtime/OpenRegStream.cpp (pool, current stream per
//               thread and device, default stream = id 0)
//   hooks       csrc/runtime/OpenRegHooks.h:16-105
//   aten ops    csrc/aten/OpenRegMinimal.cpp:150-167 (empty, as_strided,
//               view, _copy_from, _local_scalar_dense, record_stream, ...),
//               csrc/aten/ops/mm.cpp:115-120, unary_out.cpp:817-836,
//               binary_out.cpp:757-828
//   custom ops  TORCH_LIBRARY(mcpu) of csrc/aten/OpenRegExtra.cpp:147-162,
//               extended by fragment with grouped_topk / silu_and_mul /
//               rms_norm
// There is no CPU fallback: an aten op without a registration here raises
// NotImplementedError for the mcpu device.
#include <ATen/ATen.h>
#include <ATen/EmptyTensor.h>
#include <ATen/core/op_registration/adaption.h>
#include <ATen/detail/PrivateUse1HooksInterface.h>
#include <ATen/native/Resize.h>
#include <ATen/ops/as_strided_native.h>
#include <ATen/ops/view_native.h>
#include <ATen/ops/_reshape_alias_native.h>
#include <c10/core/Allocator.h>
#include <c10/core/impl/DeviceGuardImplInterface.h>
#include <c10/util/Exception.h>
#include <torch/library.h>

#include <array>
#include <atomic>
#include <mutex>
#include <unordered_set>
#include <vector>

#include "mcpu_ops.h"
#include "openreg.h"
#include "mcpu_torch.h"

namespace mcpu_torch {

#define MCPU_TORCH_CHECK(expr, what)                                                  \
  do {                                                                                \
    orError_t _e = (expr);                                                            \
    TORCH_CHECK(_e == orSuccess, what, " failed: ", mcpuGetLastErrorString());        \
  } while (0)

constexpr int kMaxDevices = 64;

// ------------------------------------------------------------------ streams
struct StreamTable {
  std::mutex mu;
  std::array<std::vector<orStream_t>, kMaxDevices> streams;  // id -> stream; 0 = default
};

static StreamTable& table() {
  static StreamTable t;
  return t;
}

static thread_local std::array<int64_t, kMaxDevices> tl_current = [] {
  std::array<int64_t, kMaxDevices> a;
  a.fill(0);
  return a;
}();

c10::DeviceIndex current_device();

// A device given without an index ("mcpu") means the current device.
static c10::DeviceIndex norm_index(c10::DeviceIndex d) {
  if (d < 0) d = current_device();
  TORCH_CHECK(d >= 0 && d < kMaxDevices, "mcpu: device index ", static_cast<int>(d), " out of range");
  return d;
}

static orStream_t create_stream(int priority) {
  orStream_t s = nullptr;
  MCPU_TORCH_CHECK(orStreamCreateWithPriority(&s, orStreamDefault, priority), "orStreamCreateWithPriority");
  return s;
}

static void ensure_default(c10::DeviceIndex dev) {
  dev = norm_index(dev);
  auto& t = table();
  std::lock_guard<std::mutex> g(t.mu);
  if (t.streams[dev].empty()) {
    int prev = 0;
    orGetDevice(&prev);
    orSetDevice(dev);
    t.streams[dev].push_back(create_stream(1));
    orSetDevice(prev);
  }
}

orStream_t stream_handle(const c10::Stream& s) {
  const c10::DeviceIndex dev = norm_index(s.device_index());
  ensure_default(dev);
  auto& t = table();
  std::lock_guard<std::mutex> g(t.mu);
  TORCH_CHECK(s.id() >= 0 && s.id() < static_cast<int64_t>(t.streams[dev].size()),
              "unknown mcpu stream id ", s.id());
  return t.streams[dev][s.id()];
}

c10::DeviceIndex current_device() {
  int d = 0;
  MCPU_TORCH_CHECK(orGetDevice(&d), "orGetDevice");
  return static_cast<c10::DeviceIndex>(d);
}

c10::Stream current_stream(c10::DeviceIndex dev) {
  dev = norm_index(dev);
  ensure_default(dev);
  return c10::Stream(c10::Stream::UNSAFE, c10::Device(c10::DeviceType::PrivateUse1, dev), tl_current[dev]);
}

orStream_t current_stream_handle(c10::DeviceIndex dev) { return stream_handle(current_stream(dev)); }

static c10::Stream new_stream(c10::DeviceIndex dev, int priority) {
  dev = norm_index(dev);
  ensure_default(dev);
  int prev = 0;
  orGetDevice(&prev);
  orSetDevice(dev);
  orStream_t s = create_stream(priority < 0 ? 0 : 1);
  orSetDevice(prev);
  auto& t = table();
  std::lock_guard<std::mutex> g(t.mu);
  t.streams[dev].push_back(s);
  return c10::Stream(c10::Stream::UNSAFE, c10::Device(c10::DeviceType::PrivateUse1, dev),
                     static_cast<int64_t>(t.streams[dev].size() - 1));
}

static void set_current_stream(const c10::Stream& s) { tl_current[norm_index(s.device_index())] = s.id(); }

// ------------------------------------------------------------------ allocator
struct Block {
  void* ptr;
  size_t size;
  c10::DeviceIndex device;
  orStream_t stream;                       // allocation stream
  std::unordered_set<orStream_t> uses;     // other streams (record_stream)
};

struct Stats {
  std::atomic<int64_t> allocated{0}, peak{0}, alloc_count{0}, free_count{0};
};
static std::array<Stats, kMaxDevices> g_stats;

static void free_block(void* ctx) {
  auto* b = static_cast<Block*>(ctx);
  if (!b) return;
  int prev = 0;
  orGetDevice(&prev);
  if (prev != b->device) orSetDevice(b->device);
  for (orStream_t u : b->uses) {
    // the memory may be reused on the allocation stream only after every
    // stream that used it has finished with it
    orEvent_t ev = nullptr;
    if (orEventCreate(&ev) == orSuccess) {
      orEventRecord(ev, u);
      orStreamWaitEvent(b->stream, ev, 0);
      orEventDestroy(ev);
    }
  }
  orFreeAsync(b->ptr, b->stream);
  if (prev != b->device) orSetDevice(prev);
  g_stats[b->device].allocated -= static_cast<int64_t>(b->size);
  g_stats[b->device].free_count++;
  delete b;
}

struct McpuAllocator final : c10::Allocator {
  c10::DataPtr allocate(size_t n) override {
    const c10::DeviceIndex dev = current_device();
    orStream_t st = current_stream_handle(dev);
    void* p = nullptr;
    if (n > 0) MCPU_TORCH_CHECK(orMallocAsync(&p, n, st), "mcpu allocation");
    auto* b = new Block{p, n, dev, st, {}};
    auto& s = g_stats[dev];
    const int64_t now = (s.allocated += static_cast<int64_t>(n));
    int64_t pk = s.peak.load();
    while (now > pk && !s.peak.compare_exchange_weak(pk, now)) {
    }
    s.alloc_count++;
    return {p, b, &free_block, c10::Device(c10::DeviceType::PrivateUse1, dev)};
  }
  c10::DeleterFnPtr raw_deleter() const override { return nullptr; }
  void copy_data(void* dst, const void* src, std::size_t count) const override {
    MCPU_TORCH_CHECK(orMemcpy(dst, src, count, orMemcpyDeviceToDevice), "mcpu copy_data");
  }
};

static McpuAllocator g_allocator;
c10::Allocator* allocator() { return &g_allocator; }

void record_stream(const c10::DataPtr& dp, const c10::Stream& s) {
  auto* b = static_cast<Block*>(dp.get_context());
  if (!b || dp.get_deleter() != &free_block) return;
  orStream_t h = stream_handle(s);
  if (h != b->stream) b->uses.insert(h);
}

MemoryStats memory_stats(c10::DeviceIndex dev) {
  auto& s = g_stats[dev];
  return {s.allocated.load(), s.peak.load(), s.alloc_count.load(), s.free_count.load()};
}

void reset_peak(c10::DeviceIndex dev) { g_stats[dev].peak = g_stats[dev].allocated.load(); }

// ------------------------------------------------------------------ pinned host memory
static void free_host(void* p) { orFreeHost(p); }

struct HostAllocator final : c10::Allocator {
  c10::DataPtr allocate(size_t n) override {
    void* p = nullptr;
    if (n > 0) MCPU_TORCH_CHECK(orMallocHost(&p, n), "orMallocHost");
    return {p, p, &free_host, c10::Device(c10::DeviceType::CPU)};
  }
  c10::DeleterFnPtr raw_deleter() const override { return &free_host; }
  void copy_data(void* dst, const void* src, std::size_t count) const override {
    std::memcpy(dst, src, count);
  }
};
static HostAllocator g_host_allocator;

// ------------------------------------------------------------------ guard
struct McpuGuardImpl final : c10::impl::DeviceGuardImplInterface {
  static constexpr c10::DeviceType static_type = c10::DeviceType::PrivateUse1;
  c10::DeviceType type() const override { return static_type; }
  c10::Device exchangeDevice(c10::Device d) const override {
    const c10::Device old = getDevice();
    if (old.index() != d.index()) setDevice(d);
    return old;
  }
  c10::Device getDevice() const override { return c10::Device(static_type, current_device()); }
  void setDevice(c10::Device d) const override {
    if (d.index() >= 0) MCPU_TORCH_CHECK(orSetDevice(d.index()), "orSetDevice");
  }
  void uncheckedSetDevice(c10::Device d) const noexcept override {
    if (d.index() >= 0) orSetDevice(d.index());
  }
  c10::Stream getStream(c10::Device d) const override { return current_stream(d.index()); }
  c10::Stream getDefaultStream(c10::Device d) const override {
    const c10::DeviceIndex i = norm_index(d.index());
    ensure_default(i);
    return c10::Stream(c10::Stream::UNSAFE, c10::Device(static_type, i), 0);
  }
  c10::Stream getNewStream(c10::Device d, int priority) const override { return new_stream(d.index(), priority); }
  c10::Stream getStreamFromGlobalPool(c10::Device d, bool high) const override {
    return new_stream(d.index(), high ? -1 : 0);
  }
  c10::Stream exchangeStream(c10::Stream s) const override {
    const c10::Stream old = current_stream(norm_index(s.device_index()));
    set_current_stream(s);
    return old;
  }
  c10::DeviceIndex deviceCount() const noexcept override {
    int n = 0;
    if (orGetDeviceCount(&n) != orSuccess) return 0;
    return static_cast<c10::DeviceIndex>(n);
  }
  void record(void** event, const c10::Stream& stream, const c10::DeviceIndex device_index,
              const c10::EventFlag flag) const override {
    TORCH_CHECK(device_index == -1 || stream.device_index() == -1 || device_index == stream.device_index(),
                "event device does not match the stream's device");
    if (!*event) {
      orEvent_t e = nullptr;
      // PYTORCH_DEFAULT: no timing; BACKEND_DEFAULT: timing enabled
      const unsigned f = flag == c10::EventFlag::PYTORCH_DEFAULT ? orEventDisableTiming : orEventEnableTiming;
      MCPU_TORCH_CHECK(orEventCreateWithFlags(&e, f), "orEventCreateWithFlags");
      *event = e;
    }
    MCPU_TORCH_CHECK(orEventRecord(static_cast<orEvent_t>(*event), stream_handle(stream)), "orEventRecord");
  }
  void block(void* event, const c10::Stream& stream) const override {
    if (!event) return;
    MCPU_TORCH_CHECK(orStreamWaitEvent(stream_handle(stream), static_cast<orEvent_t>(event), 0),
                     "orStreamWaitEvent");
  }
  bool queryEvent(void* event) const override {
    if (!event) return true;
    const orError_t e = orEventQuery(static_cast<orEvent_t>(event));
    TORCH_CHECK(e == orSuccess || e == orErrorNotReady, "orEventQuery failed: ", mcpuGetLastErrorString());
    return e == orSuccess;
  }
  void destroyEvent(void* event, const c10::DeviceIndex) const noexcept override {
    if (event) orEventDestroy(static_cast<orEvent_t>(event));
  }
  bool queryStream(const c10::Stream& s) const override {
    const orError_t e = orStreamQuery(stream_handle(s));
    TORCH_CHECK(e == orSuccess || e == orErrorNotReady, "orStreamQuery failed: ", mcpuGetLastErrorString());
    return e == orSuccess;
  }
  void synchronizeStream(const c10::Stream& s) const override {
    MCPU_TORCH_CHECK(orStreamSynchronize(stream_handle(s)), "orStreamSynchronize");
  }
  void synchronizeEvent(void* event) const override {
    if (event) MCPU_TORCH_CHECK(orEventSynchronize(static_cast<orEvent_t>(event)), "orEventSynchronize");
  }
  void synchronizeDevice(const c10::DeviceIndex) const override {
    MCPU_TORCH_CHECK(orDeviceSynchronize(), "orDeviceSynchronize");
  }
  void recordDataPtrOnStream(const c10::DataPtr& dp, const c10::Stream& s) const override {
    record_stream(dp, s);
  }
  double elapsedTime(void* e1, void* e2, const c10::DeviceIndex) const override {
    float ms = 0.0f;
    MCPU_TORCH_CHECK(orEventElapsedTime(&ms, static_cast<orEvent_t>(e1), static_cast<orEvent_t>(e2)),
                     "orEventElapsedTime");
    return ms;
  }
};

C10_REGISTER_GUARD_IMPL(PrivateUse1, McpuGuardImpl);

// ------------------------------------------------------------------ hooks
struct McpuHooks final : at::PrivateUse1HooksInterface {
  bool hasPrimaryContext(c10::DeviceIndex) const override { return true; }
  bool isAvailable() const override {
    int n = 0;
    return orGetDeviceCount(&n) == orSuccess && n > 0;
  }
  c10::DeviceIndex deviceCount() const override {
    int n = 0;
    return orGetDeviceCount(&n) == orSuccess ? static_cast<c10::DeviceIndex>(n) : 0;
  }
  void setCurrentDevice(c10::DeviceIndex d) const override { orSetDevice(d); }
  c10::DeviceIndex getCurrentDevice() const override { return current_device(); }
  c10::DeviceIndex exchangeDevice(c10::DeviceIndex d) const override {
    const c10::DeviceIndex old = current_device();
    if (old != d) orSetDevice(d);
    return old;
  }
  c10::DeviceIndex maybeExchangeDevice(c10::DeviceIndex d) const override { return exchangeDevice(d); }
  bool isPinnedPtr(const void* data) const override {
    orPointerAttributes a;
    return orPointerGetAttributes(&a, data) == orSuccess && a.type == orMemoryTypeHost;
  }
  c10::Allocator* getPinnedMemoryAllocator() const override { return &g_host_allocator; }
  const at::Generator& getDefaultGenerator(c10::DeviceIndex) const override {
    // the mcpu device draws random numbers on the host (inputs are created
    // on the CPU and copied), like the reference's CPU-generator subclass
    return at::detail::getDefaultCPUGenerator();
  }
  at::Device getDeviceFromPtr(void* data) const override {
    orPointerAttributes a;
    MCPU_TORCH_CHECK(orPointerGetAttributes(&a, data), "orPointerGetAttributes");
    return at::Device(c10::DeviceType::PrivateUse1, static_cast<c10::DeviceIndex>(a.device));
  }
};

static bool register_hooks() {
  static McpuHooks hooks;
  at::RegisterPrivateUse1HooksInterface(&hooks);
  c10::SetAllocator(c10::DeviceType::PrivateUse1, &g_allocator);
  return true;
}
static bool g_hooks_registered = register_hooks();

}  // namespace mcpu_torch
