/*
 * The reference's kernel-timing header path (include/runtime/
 * McpuKernelTiming.h of kzwrime/torch_mcpu): at::mcpu::kernel_timing and
 * the MCPU_KERNEL_TIMING_SCOPE macros are declared in mcpu_launch.h.
 */
#pragma once

#include "../mcpu_launch.h"
