/*
 * The reference's launch header path (include/runtime/McpuKernelLaunch.h of
 * kzwrime/torch_mcpu), which out-of-tree op files include as
 * <runtime/McpuKernelLaunch.h>: the B200 launch API lives in mcpu_launch.h.
 */
#pragma once

#include "../mcpu_launch.h"
