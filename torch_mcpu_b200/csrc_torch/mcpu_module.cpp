// Python module of the mcpu device (torch_mcpu_b200._C): the method table of
// the reference's torch_mcpu/csrc/Module.cpp:331-361 that the device module
// (torch.mcpu.*) and the distributed registration use.
#include <torch/csrc/utils/pybind.h>
#include <torch/extension.h>

#include "mcpu_launch.h"
#include "mcpu_torch.h"

namespace mcpu_torch {
void bind_distributed(pybind11::module& m);
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  using namespace mcpu_torch;
  namespace py = pybind11;
  m.def("_get_device_count", [] {
    int n = 0;
    return orGetDeviceCount(&n) == orSuccess ? n : 0;
  });
  m.def("_get_device", [] { return static_cast<int>(current_device()); });
  m.def("_set_device", [](int d) {
    TORCH_CHECK(orSetDevice(d) == orSuccess, "set_device: ", mcpuGetLastErrorString());
  });
  m.def("_synchronize", [](int d) {
    py::gil_scoped_release nogil;
    int prev = 0;
    orGetDevice(&prev);
    if (d >= 0) orSetDevice(d);
    const orError_t e = orDeviceSynchronize();
    if (d >= 0) orSetDevice(prev);
    TORCH_CHECK(e == orSuccess, "synchronize: ", mcpuGetLastErrorString());
  });
  m.def("_current_stream_handle", [](int d) {
    return reinterpret_cast<uintptr_t>(current_stream_handle(static_cast<c10::DeviceIndex>(d)));
  });
  m.def("_stream_handle", [](int64_t id, int d) {
    return reinterpret_cast<uintptr_t>(stream_handle(
        c10::Stream(c10::Stream::UNSAFE, c10::Device(c10::DeviceType::PrivateUse1, d), id)));
  });
  m.def("_memory_stats", [](int d) {
    const MemoryStats s = memory_stats(static_cast<c10::DeviceIndex>(d));
    py::dict r;
    r["allocated_bytes.all.current"] = s.allocated;
    r["allocated_bytes.all.peak"] = s.peak;
    r["allocation.all.allocated"] = s.alloc_count;
    r["allocation.all.freed"] = s.free_count;
    return r;
  });
  m.def("_reset_peak_memory_stats", [](int d) { reset_peak(static_cast<c10::DeviceIndex>(d)); });
  m.def("_empty_cache", [] {
    TORCH_CHECK(orMemPoolTrim(0) == orSuccess, "empty_cache: ", mcpuGetLastErrorString());
  });
  m.def("_get_default_stream", [](int d) {
    // stream id 0 of every device is its default stream
    return py::make_tuple(0, d, static_cast<int>(c10::DeviceType::PrivateUse1));
  });
  m.def("_mem_get_info", [](int d) {
    size_t free_b = 0, total_b = 0;
    TORCH_CHECK(mcpu_mem_get_info(d, &free_b, &total_b) == orSuccess, "mem_get_info: ",
                mcpuGetLastErrorString());
    return py::make_tuple(free_b, total_b);
  });
  m.def("_mem_pool_reserved", [](int d) {
    uint64_t cur = 0, peak = 0;
    TORCH_CHECK(mcpu_mem_pool_reserved(d, &cur, &peak) == orSuccess, "memory_reserved: ",
                mcpuGetLastErrorString());
    return py::make_tuple(cur, peak);
  });
  // CUDA graphs of the work enqueued on the current mcpu stream
  m.def("_graph_begin", [](int d) {
    TORCH_CHECK(mcpu_graph_capture_begin(current_stream_handle(static_cast<c10::DeviceIndex>(d))) == orSuccess,
                "graph capture: ", mcpuGetLastErrorString());
  });
  m.def("_graph_end", [](int d) {
    void* exec = nullptr;
    TORCH_CHECK(mcpu_graph_capture_end(current_stream_handle(static_cast<c10::DeviceIndex>(d)), &exec) == orSuccess,
                "graph capture: ", mcpuGetLastErrorString());
    return reinterpret_cast<uintptr_t>(exec);
  });
  m.def("_graph_replay", [](uintptr_t exec, int d) {
    TORCH_CHECK(mcpu_graph_launch(reinterpret_cast<void*>(exec),
                                  current_stream_handle(static_cast<c10::DeviceIndex>(d))) == orSuccess,
                "graph replay: ", mcpuGetLastErrorString());
  });
  m.def("_graph_destroy", [](uintptr_t exec) {
    TORCH_CHECK(mcpu_graph_destroy(reinterpret_cast<void*>(exec)) == orSuccess, "graph destroy: ",
                mcpuGetLastErrorString());
  });
  // kernel timing of the launch API (include/mcpu_launch.h)
  m.def("_set_kernel_timing_enabled", [](bool on) { at::mcpu::kernel_timing::set_enabled(on); });
  m.def("_reset_kernel_timing", [] { at::mcpu::kernel_timing::reset(); });
  m.def("_get_kernel_timing", [] {
    py::list out;
    for (const auto& snap : at::mcpu::kernel_timing::snapshot()) {
      py::list events;
      for (const auto& e : snap.events) {
        py::dict ev;
        ev["name"] = e.name ? e.name : "";
        ev["stream"] = e.stream;
        ev["begin_time"] = e.begin_time;
        ev["end_time"] = e.end_time;
        ev["elapsed_time"] = static_cast<double>(static_cast<int64_t>(e.end_time - e.begin_time)) / 1000.0;
        events.append(ev);
      }
      py::dict d;
      d["role"] = snap.role;
      d["events"] = events;
      out.append(d);
    }
    return out;
  });
  bind_distributed(m);
}
