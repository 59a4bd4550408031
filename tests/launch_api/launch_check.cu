// A caller of the mcpu kernel-launch API (include/mcpu_launch.h), written the
// way the reference's op files use McpuKernelLaunch.h: host callables,
// MCPU_LAUNCH_TIMED_KERNEL, the tensor-selected stream, and the B200 overload
// that launches a __global__ function.  Built as a small Python module for
// tests/test_launch_api_gpu.py.
#include <torch/extension.h>

#include <mutex>
#include <vector>

#include "mcpu_launch.h"

namespace {

__global__ void fill_kernel(float* p, long long n, float v) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) p[i] = v + static_cast<float>(i);
}

std::mutex g_mu;
std::vector<int64_t> g_trace;

void note(int64_t v) {
  std::lock_guard<std::mutex> lk(g_mu);
  g_trace.push_back(v);
}

// Host tasks in stream order, interleaved with a device kernel.
std::vector<int64_t> host_tasks(const at::Tensor& t) {
  {
    std::lock_guard<std::mutex> lk(g_mu);
    g_trace.clear();
  }
  at::mcpu::launch_kernel([] { note(1); });
  at::mcpu::launch_kernel(t, [] { note(2); });
  const long long n = t.numel();
  at::mcpu::launch_kernel(fill_kernel, dim3((n + 255) / 256), dim3(256), 0,
                          c10::mcpu::getCurrentMcpuStream(), t.data_ptr<float>(), n, 10.0f);
  int captured = 3;
  MCPU_LAUNCH_TIMED_KERNEL("launch_check.timed", ([captured]), { note(captured); });
  TORCH_CHECK(orLaunchKernel(c10::mcpu::getCurrentMcpuStream(), [](int v) { note(v); }, 4) == orSuccess);
  TORCH_CHECK(orStreamSynchronize(c10::mcpu::getCurrentMcpuStream()) == orSuccess);
  std::lock_guard<std::mutex> lk(g_mu);
  return g_trace;
}

void device_fill(const at::Tensor& t, double v, bool timed) {
  TORCH_CHECK(t.device().type() == c10::DeviceType::PrivateUse1 && t.is_contiguous() &&
              t.scalar_type() == at::kFloat);
  const long long n = t.numel();
  orStream_t s = at::mcpu::detail::get_kernel_launch_stream(t);
  if (timed)
    at::mcpu::launch_timed_kernel_on_stream(s, "launch_check.fill", fill_kernel, dim3((n + 255) / 256),
                                            dim3(256), 0, t.data_ptr<float>(), n, static_cast<float>(v));
  else
    at::mcpu::launch_kernel(fill_kernel, dim3((n + 255) / 256), dim3(256), 0, s, t.data_ptr<float>(), n,
                            static_cast<float>(v));
}

std::vector<double> timing(bool enable, bool reset) {
  namespace kt = at::mcpu::kernel_timing;
  kt::set_enabled(enable);
  if (reset) kt::reset();
  const auto n = kt::event_count();
  std::vector<double> r{static_cast<double>(n)};
  if (n > 0) r.push_back(kt::elapsed_us_between(0, n));
  return r;
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("host_tasks", &host_tasks);
  m.def("device_fill", &device_fill);
  m.def("timing", &timing);
}
