// Declarations shared by the PyTorch-facing sources of the mcpu device.
#pragma once

#include <c10/core/Allocator.h>
#include <c10/core/Stream.h>

#include "mcpu_ops.h"
#include "openreg.h"

namespace mcpu_torch {

c10::DeviceIndex current_device();
c10::Stream current_stream(c10::DeviceIndex dev);
orStream_t stream_handle(const c10::Stream& s);
orStream_t current_stream_handle(c10::DeviceIndex dev);
c10::Allocator* allocator();
void record_stream(const c10::DataPtr& dp, const c10::Stream& s);

struct MemoryStats {
  int64_t allocated, peak, alloc_count, free_count;
};
MemoryStats memory_stats(c10::DeviceIndex dev);
void reset_peak(c10::DeviceIndex dev);

}  // namespace mcpu_torch
