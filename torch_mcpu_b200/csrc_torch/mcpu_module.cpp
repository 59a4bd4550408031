// Python module of the mcpu device (torch_mcpu_b200._C): the method table of
// the reference's torch_mcpu/csrc/Module.cpp:331-361 that the device module
// (torch.mcpu.*) and the distributed registration use.
#include <torch/csrc/utils/pybind.h>
#include <torch/extension.h>

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
  bind_distributed(m);
}
