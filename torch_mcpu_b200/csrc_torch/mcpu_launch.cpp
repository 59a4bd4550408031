// Exported side of the kernel-launch API (include/mcpu_launch.h): the
// kernel-timing log, the memory-guard hooks (no-ops on B200: device memory
// carries no host-side protection) and the stream lookups.  Mirrors
// csrc/runtime/McpuKernelLaunch.cpp and McpuKernelTiming.cpp of
// kzwrime/torch_mcpu.
#include <array>
#include <memory>

#include "mcpu_launch.h"
#include "mcpu_torch.h"

namespace c10::mcpu {
orStream_t getCurrentMcpuStream(c10::DeviceIndex device) {
  if (device < 0) device = mcpu_torch::current_device();
  return mcpu_torch::current_stream_handle(device);
}
}  // namespace c10::mcpu

namespace at::mcpu::kernel_timing {

namespace {
constexpr std::size_t kCapacity = 262144;
std::unique_ptr<std::array<Event, kCapacity>> g_log;
std::atomic<std::size_t> g_next{0};
}  // namespace

std::atomic<bool> g_enabled{false};

void set_enabled(bool value) {
  if (value && !g_log) g_log = std::make_unique<std::array<Event, kCapacity>>();
  g_enabled.store(value, std::memory_order_relaxed);
}

void reset() { g_next.store(0, std::memory_order_relaxed); }

Event* reserve_event_slot(const char* name, std::uint64_t stream) {
  if (!enabled() || !g_log) return nullptr;
  const std::size_t i = g_next.fetch_add(1, std::memory_order_relaxed);
  if (i >= kCapacity) return nullptr;
  Event& e = (*g_log)[i];
  e = Event{name, stream, 0, 0};
  return &e;
}

std::size_t event_count() {
  const std::size_t n = g_next.load(std::memory_order_relaxed);
  return n < kCapacity ? n : kCapacity;
}

double elapsed_us_between(std::size_t begin, std::size_t end) {
  const std::size_t n = event_count();
  TORCH_CHECK(begin < end && end <= n, "kernel_timing: bad event range [", begin, ", ", end, ") of ", n);
  const Event& a = (*g_log)[begin];
  const Event& b = (*g_log)[end - 1];
  return static_cast<double>(static_cast<int64_t>(b.end_time - a.begin_time)) / 1000.0;
}

std::vector<ThreadSnapshot> snapshot() {
  std::vector<ThreadSnapshot> out;
  const std::size_t n = event_count();
  if (n == 0) return out;
  out.push_back(ThreadSnapshot{"worker", std::vector<Event>(g_log->begin(), g_log->begin() + n)});
  return out;
}

}  // namespace at::mcpu::kernel_timing

namespace at::mcpu::detail {

bool enter_kernel_task() { return false; }
void exit_kernel_task(bool) noexcept {}
void protect_memory(void*) noexcept {}
void unprotect_memory(const void*, std::unordered_set<void*>&) {}
void unprotect_tensor_memory(const at::TensorBase&, std::unordered_set<void*>&) {}
void unprotect_all_device_memory(std::unordered_set<void*>&) {}

orStream_t get_kernel_launch_stream(const at::Tensor& stream_tensor) {
  TORCH_CHECK(stream_tensor.defined() && stream_tensor.device().type() == c10::DeviceType::PrivateUse1,
              "launch_kernel expects an mcpu tensor to select the stream");
  return mcpu_torch::current_stream_handle(stream_tensor.device().index());
}

}  // namespace at::mcpu::detail
