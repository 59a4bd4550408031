// Compile-only check of the launch API through the reference's header paths
// (<runtime/McpuKernelLaunch.h>, <runtime/McpuKernelTiming.h>): every form an
// out-of-tree op file uses, instantiated once.  Host callables here touch no
// device memory, as the B200 launch API requires.
#include <ATen/ATen.h>
#include <runtime/McpuKernelLaunch.h>
#include <runtime/McpuKernelTiming.h>

#include <atomic>
#include <memory>

namespace {

std::atomic<int> g_runs{0};

__attribute__((unused)) void every_form(const at::Tensor& t, orStream_t s) {
  at::mcpu::launch_kernel(t, [t]() mutable {
    at::mcpu::KernelMemoryGuard guard(t);
    g_runs.fetch_add(1);
  });
  at::mcpu::launch_kernel(t, "check.named", [] { g_runs.fetch_add(1); });
  at::mcpu::launch_kernel([] { g_runs.fetch_add(1); }, s);
  at::mcpu::launch_timed_kernel("check.timed", [](at::mcpu::kernel_timing::Event* ev) mutable {
    MCPU_KERNEL_TIMING_SCOPE_EVENT("check.timed", ev);
    g_runs.fetch_add(1);
  });
  auto payload = std::make_unique<int>(3);
  at::mcpu::launch_timed_kernel_on_stream(s, "check.move_only",
                                          [p = std::move(payload)](at::mcpu::kernel_timing::Event*) mutable {
                                            *p += 1;
                                          });
  int captured = 5;
  MCPU_LAUNCH_TIMED_KERNEL("check.macro", ([captured]), { g_runs.fetch_add(captured); });
  TORCH_CHECK(orLaunchKernel(s, [](int v) { g_runs.fetch_add(v); }, 2) == orSuccess);
  TORCH_CHECK(orLaunchKernelNamed(s, "check.or", [] {}) == orSuccess);
  at::mcpu::KernelPointerMemoryGuard pg({t.const_data_ptr()});
  at::mcpu::KernelAllMemoryGuard ag;
  at::mcpu::kernel_timing::set_enabled(true);
  at::mcpu::kernel_timing::reset();
  (void)at::mcpu::kernel_timing::event_count();
  (void)at::mcpu::kernel_timing::snapshot();
  (void)c10::mcpu::getCurrentMcpuStream();
  (void)at::mcpu::detail::get_kernel_launch_stream(t);
}

}  // namespace
