// The reference's TORCH_LIBRARY(mcpu) block (csrc/aten/OpenRegExtra.cpp:
// 147-162 of kzwrime/torch_mcpu) with its six schemas unchanged, and their
// mcpu implementations on B200 (reference bodies: csrc/aten/native/
// Extra.cpp:251-353).  The hot-path ops join the namespace as a fragment
// (mcpu_aten.cpp).
//
// stream_sleep_fill_ / stream_sleep_copy_ enqueue a device kernel that
// waits on the GPU timer, then fills / copies (the reference sleeps on its
// worker thread); first_element_int reads element 0 at once, without
// waiting for queued work, as the reference reads host memory directly.
// kernel_launch_lifetime_counts / kernel_launch_failed_lifetime_counts run
// the launch API's host tasks with a move-only payload and report how many
// payloads were constructed, destroyed and run.
#include <ATen/ATen.h>
#include <torch/library.h>

#include <atomic>
#include <memory>
#include <tuple>

#include "mcpu_launch.h"
#include "mcpu_torch.h"

namespace mcpu_torch {
namespace {

void check_ok(orError_t e, const char* what) {
  TORCH_CHECK(e == orSuccess, what, ": ", mcpuGetLastErrorString());
}

void check_stream_test_tensor(const at::Tensor& t) {
  TORCH_CHECK(t.device().type() == c10::DeviceType::PrivateUse1, "stream test ops expect mcpu tensors");
  TORCH_CHECK(t.scalar_type() == at::kLong, "stream test ops only support int64 tensors");
  TORCH_CHECK(t.is_contiguous(), "stream test ops require contiguous input");
  TORCH_CHECK(t.numel() > 0, "stream test ops require non-empty input");
}

// Host stamps around a device launch when kernel timing is on (the
// reference's launch_timed_kernel records the same span for its lambda).
template <typename Launch>
void timed(orStream_t s, const char* name, Launch&& launch) {
  auto* slot = at::mcpu::kernel_timing::reserve_event_slot(
      name, static_cast<std::uint64_t>(reinterpret_cast<std::uintptr_t>(s)));
  if (slot) {
    TORCH_CHECK(orLaunchKernel(s, [slot, name] {
                  slot->name = name;
                  slot->begin_time = at::mcpu::kernel_timing::read_timer();
                }) == orSuccess,
                "orLaunchKernel failed");
  }
  launch();
  if (slot) {
    TORCH_CHECK(orLaunchKernel(s, [slot] { slot->end_time = at::mcpu::kernel_timing::read_timer(); }) ==
                    orSuccess,
                "orLaunchKernel failed");
  }
}

at::Tensor custom_abs(at::Tensor x) { return at::abs(x); }

at::Tensor& stream_sleep_fill_(at::Tensor& x, int64_t value, int64_t sleep_ms) {
  check_stream_test_tensor(x);
  const orStream_t s = current_stream_handle(x.device().index());
  timed(s, "mcpu::stream_sleep_fill_", [&] {
    check_ok(mcpu_stream_sleep_fill_i64(x.data_ptr<int64_t>(), x.numel(), value, sleep_ms, s),
             "stream_sleep_fill_");
  });
  return x;
}

at::Tensor& stream_sleep_copy_(at::Tensor& dst, const at::Tensor& src, int64_t sleep_ms) {
  check_stream_test_tensor(dst);
  check_stream_test_tensor(src);
  TORCH_CHECK(dst.sizes() == src.sizes(), "stream_sleep_copy_ expects src/dst with identical shapes");
  const orStream_t s = current_stream_handle(dst.device().index());
  check_ok(mcpu_stream_sleep_copy_i64(dst.data_ptr<int64_t>(), src.const_data_ptr<int64_t>(), dst.numel(),
                                      sleep_ms, s),
           "stream_sleep_copy_");
  return dst;
}

int64_t first_element_int(const at::Tensor& x) {
  check_stream_test_tensor(x);
  int64_t v = 0;
  check_ok(mcpu_read_i64_now(x.const_data_ptr<int64_t>(), &v), "first_element_int");
  return v;
}

std::atomic<int64_t> g_constructed{0}, g_destroyed{0}, g_ran{0};

struct LifetimePayload {
  explicit LifetimePayload(int64_t v) : value(v) { g_constructed.fetch_add(1, std::memory_order_relaxed); }
  ~LifetimePayload() { g_destroyed.fetch_add(1, std::memory_order_relaxed); }
  int64_t value;
};

void reset_counts() {
  g_constructed.store(0, std::memory_order_relaxed);
  g_destroyed.store(0, std::memory_order_relaxed);
  g_ran.store(0, std::memory_order_relaxed);
}

std::tuple<int64_t, int64_t, int64_t> counts() {
  return std::make_tuple(g_constructed.load(std::memory_order_relaxed), g_destroyed.load(std::memory_order_relaxed),
                         g_ran.load(std::memory_order_relaxed));
}

std::tuple<int64_t, int64_t, int64_t> kernel_launch_lifetime_counts(const at::Tensor& stream_selector,
                                                                    int64_t launches) {
  check_stream_test_tensor(stream_selector);
  TORCH_CHECK(launches >= 0, "launches must be non-negative");
  reset_counts();
  for (int64_t i = 0; i < launches; ++i) {
    auto payload = std::make_unique<LifetimePayload>(i);
    at::mcpu::launch_timed_kernel(
        "mcpu::kernel_launch_lifetime_counts",
        [payload = std::move(payload)](at::mcpu::kernel_timing::Event* timing_event) mutable {
          MCPU_KERNEL_TIMING_SCOPE_EVENT("mcpu::kernel_launch_lifetime_counts", timing_event);
          g_ran.fetch_add(1, std::memory_order_relaxed);
          payload->value += 1;
        });
  }
  check_ok(orStreamSynchronize(current_stream_handle(stream_selector.device().index())),
           "kernel_launch_lifetime_counts");
  return counts();
}

std::tuple<int64_t, int64_t, int64_t> kernel_launch_failed_lifetime_counts(const at::Tensor& stream_selector) {
  check_stream_test_tensor(stream_selector);
  reset_counts();
  bool caught = false;
  try {
    auto payload = std::make_unique<LifetimePayload>(0);
    at::mcpu::launch_timed_kernel_on_stream(
        static_cast<orStream_t>(nullptr), "mcpu::kernel_launch_failed_lifetime_counts",
        [payload = std::move(payload)](at::mcpu::kernel_timing::Event* timing_event) mutable {
          MCPU_KERNEL_TIMING_SCOPE_EVENT("mcpu::kernel_launch_failed_lifetime_counts", timing_event);
          g_ran.fetch_add(1, std::memory_order_relaxed);
        });
  } catch (const c10::Error&) {
    caught = true;
  }
  TORCH_CHECK(caught, "expected null stream launch to fail");
  return counts();
}

}  // namespace
}  // namespace mcpu_torch

TORCH_LIBRARY(mcpu, m) {
  m.def("custom_abs(Tensor input)-> Tensor");
  m.def("stream_sleep_fill_(Tensor(a!) input, int value, int sleep_ms) -> Tensor(a!)");
  m.def("stream_sleep_copy_(Tensor(a!) dst, Tensor src, int sleep_ms) -> Tensor(a!)");
  m.def("first_element_int(Tensor input) -> int");
  m.def("kernel_launch_lifetime_counts(Tensor stream_selector, int launches) -> (int, int, int)");
  m.def("kernel_launch_failed_lifetime_counts(Tensor stream_selector) -> (int, int, int)");
}

TORCH_LIBRARY_IMPL(mcpu, PrivateUse1, m) {
  using namespace mcpu_torch;
  m.impl("custom_abs", &custom_abs);
  m.impl("stream_sleep_fill_", &stream_sleep_fill_);
  m.impl("stream_sleep_copy_", &stream_sleep_copy_);
  m.impl("first_element_int", &first_element_int);
  m.impl("kernel_launch_lifetime_counts", &kernel_launch_lifetime_counts);
  m.impl("kernel_launch_failed_lifetime_counts", &kernel_launch_failed_lifetime_counts);
}
