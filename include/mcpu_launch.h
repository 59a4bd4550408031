/*
 * Kernel-launch API of the mcpu device on B200 (C++ only, compiled into the
 * caller).  Source-compatible with the reference's launch helpers:
 *   MCPU_LAUNCH_TIMED_KERNEL, at::mcpu::launch_kernel / launch_timed_kernel /
 *   launch_kernel_on_stream / launch_timed_kernel_on_stream and the memory
 *   guards (include/runtime/McpuKernelLaunch.h:29-320 of kzwrime/torch_mcpu),
 *   at::mcpu::kernel_timing (include/runtime/McpuKernelTiming.h:50-60),
 *   orLaunchKernel / orLaunchKernelNamed
 *   (third_party/openreg/include/openreg.inl:238-263).
 *
 * Semantics on B200.  A host callable is enqueued with cudaLaunchHostFunc:
 * it runs on a CUDA runtime thread once the stream reaches it, in stream
 * order.  Device memory is not addressable from the host, so a host
 * callable must not touch device memory and must not call CUDA (a CUDA rule
 * for host functions); code that computed on device memory inside a host
 * lambda launches a __global__ function instead, through the overload
 *   launch_kernel(kernel, grid, block, smem, stream, args...)
 * which is an ordinary asynchronous kernel launch on `stream`.  The memory
 * guards are no-ops (device memory has no host protection to lift).
 *
 * Timing: with kernel_timing enabled, a timed host callable records host
 * clock stamps around its body; a timed __global__ launch records stamps
 * from host functions enqueued before and after the kernel (stream order),
 * so its span includes the callback latency (microseconds).
 */
#pragma once

#include <ATen/ATen.h>
#include <c10/util/ApproximateClock.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstddef>
#include <cstdint>
#include <functional>
#include <initializer_list>
#include <tuple>
#include <type_traits>
#include <unordered_set>
#include <utility>
#include <vector>

#include "openreg.h"

#define MCPU_LAUNCH_EXPORT __attribute__((visibility("default")))

namespace c10::mcpu {
/* The current mcpu stream of `device` (-1: the current device). */
MCPU_LAUNCH_EXPORT orStream_t getCurrentMcpuStream(c10::DeviceIndex device = -1);
}  // namespace c10::mcpu

/* ------------------------------------------------------------ host tasks */
namespace mcpu_launch_detail {

template <typename F, typename... A>
struct HostTask {
  F f;
  std::tuple<A...> args;
  static void run(void* p) {
    auto* t = static_cast<HostTask*>(p);
    std::apply(t->f, t->args);
    delete t;
  }
};

template <typename F, typename... Args>
inline orError_t enqueue_host(orStream_t stream, F&& f, Args&&... args) {
  using Task = HostTask<std::decay_t<F>, std::decay_t<Args>...>;
  auto* t = new Task{std::forward<F>(f), std::make_tuple(std::forward<Args>(args)...)};
  const cudaError_t e =
      cudaLaunchHostFunc(reinterpret_cast<cudaStream_t>(stream), &Task::run, t);
  if (e != cudaSuccess) {
    delete t;
    return orErrorUnknown;
  }
  return orSuccess;
}

}  // namespace mcpu_launch_detail

/* Enqueue kernel_func(args...) as a host task on `stream` (stream order). */
template <typename Func, typename... Args>
inline orError_t orLaunchKernel(orStream_t stream, Func&& kernel_func, Args&&... args) {
  if (!stream) return orErrorUnknown;
  return mcpu_launch_detail::enqueue_host(stream, std::forward<Func>(kernel_func),
                                          std::forward<Args>(args)...);
}

/* As orLaunchKernel; the name is kept for tracing by the caller. */
template <typename Func, typename... Args>
inline orError_t orLaunchKernelNamed(orStream_t stream, const char* debug_name, Func&& kernel_func,
                                     Args&&... args) {
  (void)debug_name;
  return orLaunchKernel(stream, std::forward<Func>(kernel_func), std::forward<Args>(args)...);
}

/* ---------------------------------------------------------- kernel timing */
#define MCPU_KERNEL_TIMING_CONCAT_INNER(a, b) a##b
#define MCPU_KERNEL_TIMING_CONCAT(a, b) MCPU_KERNEL_TIMING_CONCAT_INNER(a, b)
#define MCPU_KERNEL_TIMING_SCOPE(name) \
  ::at::mcpu::kernel_timing::Scope MCPU_KERNEL_TIMING_CONCAT(_mcpu_kernel_timing_scope_, __COUNTER__)(name)
#define MCPU_KERNEL_TIMING_SCOPE_EVENT(name, event)                                           \
  ::at::mcpu::kernel_timing::EventScope MCPU_KERNEL_TIMING_CONCAT(_mcpu_kernel_timing_scope_, \
                                                                  __COUNTER__)(name, event)

namespace at::mcpu::kernel_timing {

struct Event {
  const char* name;
  std::uint64_t stream;
  std::uint64_t begin_time;
  std::uint64_t end_time;
};

struct ThreadSnapshot {
  const char* role;
  std::vector<Event> events;
};

MCPU_LAUNCH_EXPORT extern std::atomic<bool> g_enabled;
MCPU_LAUNCH_EXPORT void set_enabled(bool value);
MCPU_LAUNCH_EXPORT void reset();
/* A slot for one launch (nullptr when timing is disabled or the log is full). */
MCPU_LAUNCH_EXPORT Event* reserve_event_slot(const char* name, std::uint64_t stream = 0);
MCPU_LAUNCH_EXPORT std::size_t event_count();
/* Microseconds from the begin of event `begin` to the end of event `end - 1`. */
MCPU_LAUNCH_EXPORT double elapsed_us_between(std::size_t begin, std::size_t end);
MCPU_LAUNCH_EXPORT std::vector<ThreadSnapshot> snapshot();

inline thread_local Event* current_event_slot = nullptr;

inline bool enabled() { return g_enabled.load(std::memory_order_relaxed); }
inline std::uint64_t read_timer() {
  return static_cast<std::uint64_t>(c10::getTime(/*allow_monotonic=*/true));
}

class CurrentEventSlotGuard {
 public:
  explicit CurrentEventSlotGuard(Event* slot) noexcept : previous_(current_event_slot) {
    current_event_slot = slot;
  }
  ~CurrentEventSlotGuard() noexcept { current_event_slot = previous_; }
  CurrentEventSlotGuard(const CurrentEventSlotGuard&) = delete;
  CurrentEventSlotGuard& operator=(const CurrentEventSlotGuard&) = delete;

 private:
  Event* previous_;
};

class EventScope {
 public:
  EventScope(const char* name, Event* event) noexcept : event_(event), begin_(0) {
    if (event_) {
      begin_ = read_timer();
      event_->name = name;
    }
  }
  ~EventScope() noexcept {
    if (event_) {
      event_->begin_time = begin_;
      event_->end_time = read_timer();
    }
  }
  EventScope(const EventScope&) = delete;
  EventScope& operator=(const EventScope&) = delete;

 private:
  Event* event_;
  std::uint64_t begin_;
};

class Scope : public EventScope {
 public:
  explicit Scope(const char* name) noexcept : EventScope(name, current_event_slot) {}
};

}  // namespace at::mcpu::kernel_timing

#define MCPU_LAUNCH_UNPAREN(...) __VA_ARGS__
#define MCPU_LAUNCH_TIMED_KERNEL(name, captures, ...)                                        \
  ::at::mcpu::launch_timed_kernel(                                                           \
      name, MCPU_LAUNCH_UNPAREN captures(::at::mcpu::kernel_timing::Event * timing_event) mutable { \
        MCPU_KERNEL_TIMING_SCOPE_EVENT(name, timing_event);                                  \
        __VA_ARGS__                                                                          \
      })

/* ------------------------------------------------------- guards, helpers */
namespace at::mcpu::detail {

MCPU_LAUNCH_EXPORT bool enter_kernel_task();
MCPU_LAUNCH_EXPORT void exit_kernel_task(bool previous) noexcept;
MCPU_LAUNCH_EXPORT void protect_memory(void* ptr) noexcept;
MCPU_LAUNCH_EXPORT void unprotect_memory(const void* ptr, std::unordered_set<void*>& unprotected);
MCPU_LAUNCH_EXPORT void unprotect_tensor_memory(const at::TensorBase& tensor,
                                                std::unordered_set<void*>& unprotected);
MCPU_LAUNCH_EXPORT void unprotect_all_device_memory(std::unordered_set<void*>& unprotected);
/* The current stream of the tensor's mcpu device. */
MCPU_LAUNCH_EXPORT orStream_t get_kernel_launch_stream(const at::Tensor& stream_tensor);

}  // namespace at::mcpu::detail

namespace at::mcpu {

class KernelTaskScope {
 public:
  KernelTaskScope() noexcept = default;
  KernelTaskScope(const KernelTaskScope&) = delete;
  KernelTaskScope& operator=(const KernelTaskScope&) = delete;
};

class KernelPointerMemoryGuard {
 public:
  explicit KernelPointerMemoryGuard(std::initializer_list<const void*>) noexcept {}
  explicit KernelPointerMemoryGuard(c10::ArrayRef<const void*>) noexcept {}
  KernelPointerMemoryGuard(const KernelPointerMemoryGuard&) = delete;
  KernelPointerMemoryGuard& operator=(const KernelPointerMemoryGuard&) = delete;
};

class KernelAllMemoryGuard {
 public:
  KernelAllMemoryGuard() noexcept = default;
  KernelAllMemoryGuard(const KernelAllMemoryGuard&) = delete;
  KernelAllMemoryGuard& operator=(const KernelAllMemoryGuard&) = delete;
};

class KernelMemoryGuard {
 public:
  template <typename... Args>
  explicit KernelMemoryGuard(const Args&...) noexcept {}
  KernelMemoryGuard(const KernelMemoryGuard&) = delete;
  KernelMemoryGuard& operator=(const KernelMemoryGuard&) = delete;
};

template <typename Func>
inline void launch_kernel_on_stream(orStream_t stream, Func&& func) {
  TORCH_CHECK(orLaunchKernelNamed(stream, "mcpu_kernel", std::forward<Func>(func)) == orSuccess,
              "orLaunchKernel failed");
}

template <typename Func>
inline void launch_kernel_on_stream(orStream_t stream, const char* record_name, Func&& func) {
  TORCH_CHECK(orLaunchKernelNamed(stream, record_name, std::forward<Func>(func)) == orSuccess,
              "orLaunchKernelNamed failed");
}

/* func(kernel_timing::Event*) runs as a host task; the slot is nullptr when
 * timing is off. */
template <typename Func>
inline void launch_timed_kernel_on_stream(orStream_t stream, const char* record_name, Func&& func) {
  auto* slot = kernel_timing::reserve_event_slot(
      record_name, static_cast<std::uint64_t>(reinterpret_cast<std::uintptr_t>(stream)));
  TORCH_CHECK(orLaunchKernelNamed(stream, record_name, std::forward<Func>(func), slot) == orSuccess,
              "orLaunchKernel failed");
}

template <typename Func>
inline void launch_kernel(Func&& func, orStream_t stream = c10::mcpu::getCurrentMcpuStream()) {
  launch_kernel_on_stream(stream, std::forward<Func>(func));
}

template <typename Func>
inline void launch_timed_kernel(const char* record_name, Func&& func) {
  launch_timed_kernel_on_stream(c10::mcpu::getCurrentMcpuStream(), record_name,
                                std::forward<Func>(func));
}

template <typename Func>
inline void launch_kernel(const char* record_name, Func&& func,
                          orStream_t stream = c10::mcpu::getCurrentMcpuStream()) {
  launch_kernel_on_stream(stream, record_name, std::forward<Func>(func));
}

template <typename Func>
inline void launch_kernel(const at::Tensor& stream_tensor, const char* record_name, Func&& func) {
  launch_kernel_on_stream(detail::get_kernel_launch_stream(stream_tensor), record_name,
                          std::forward<Func>(func));
}

template <typename Func>
inline void launch_kernel(const at::Tensor& stream_tensor, Func&& func) {
  launch_kernel_on_stream(detail::get_kernel_launch_stream(stream_tensor), std::forward<Func>(func));
}

/* A __global__ function on `stream`: kernel<<<grid, block, smem, stream>>>(args...).
 * The arguments are converted to the kernel's parameter types. */
template <typename... KArgs, typename... Args>
inline void launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                          orStream_t stream, Args&&... args) {
  static_assert(sizeof...(KArgs) == sizeof...(Args), "launch_kernel: argument count mismatch");
  std::tuple<KArgs...> held(std::forward<Args>(args)...);
  void* argv[sizeof...(KArgs) > 0 ? sizeof...(KArgs) : 1];
  std::apply([&](auto&... a) {
    int i = 0;
    ((argv[i++] = static_cast<void*>(&a)), ...);
  }, held);
  const cudaError_t e = cudaLaunchKernel(reinterpret_cast<const void*>(kernel), grid, block, argv,
                                         smem, reinterpret_cast<cudaStream_t>(stream));
  TORCH_CHECK(e == cudaSuccess, "mcpu kernel launch failed: ", cudaGetErrorString(e));
}

/* As above, timed: host stamps enqueued before and after the kernel. */
template <typename... KArgs, typename... Args>
inline void launch_timed_kernel_on_stream(orStream_t stream, const char* record_name,
                                          void (*kernel)(KArgs...), dim3 grid, dim3 block,
                                          size_t smem, Args&&... args) {
  auto* slot = kernel_timing::reserve_event_slot(
      record_name, static_cast<std::uint64_t>(reinterpret_cast<std::uintptr_t>(stream)));
  if (slot) {
    slot->name = record_name;
    TORCH_CHECK(orLaunchKernel(stream, [slot] { slot->begin_time = kernel_timing::read_timer(); }) ==
                    orSuccess,
                "orLaunchKernel failed");
  }
  launch_kernel(kernel, grid, block, smem, stream, std::forward<Args>(args)...);
  if (slot) {
    TORCH_CHECK(orLaunchKernel(stream, [slot] { slot->end_time = kernel_timing::read_timer(); }) ==
                    orSuccess,
                "orLaunchKernel failed");
  }
}

}  // namespace at::mcpu
