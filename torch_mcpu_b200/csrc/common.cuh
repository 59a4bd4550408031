// Shared helpers for the sm_100a kernels and the C-ABI layer.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "openreg.h"
#include "mcpu_ops.h"

namespace mcpu {

// Thread-local last-error text behind mcpuGetLastErrorString().
void set_last_error(const char* fmt, ...);

// Maps a CUDA status to orError_t, recording the CUDA message on failure.
orError_t from_cuda(cudaError_t st, const char* what);

// Raises `kernel`'s dynamic shared-memory limit to at least `bytes` on the
// current device (once per kernel, device and size; thread-safe).
cudaError_t ensure_dynamic_smem(const void* kernel, int bytes);

// Driver entry point by name (cudaGetDriverEntryPoint), or nullptr.
void* driver_entry(const char* name);

// Device error flags of the kernels with bounded waits (OR-ed, optionally reset).
namespace gemm {
orError_t read_error(int* flag, bool reset);
}
namespace router {
orError_t read_error(int* flag, bool reset);
}
namespace bw {
orError_t read_error(int* flag, bool reset);
}
orError_t aten_read_error(int* flag, bool reset);
orError_t moe_read_error(int* flag, bool reset);

// moe_align_block_size's argument check and its two launches (moe_align.cu),
// also behind the router + dispatch entry point when that is not one launch.
namespace moe {
orError_t check_args(const int32_t* topk_ids, long long numel, int E, int bs, const int32_t* sorted,
                     long long sorted_cap, const int32_t* expert_ids, long long eid_cap, const int32_t* post_pad,
                     int* nchunks_out);
orError_t launch(const int32_t* topk_ids, long long numel, int E, int bs, int32_t* sorted, long long sorted_cap,
                 int32_t* expert_ids, long long eid_cap, int32_t* post_pad, int32_t* ws, int nchunks,
                 cudaStream_t st);
}  // namespace moe
orError_t sampler_read_error(int* flag, bool reset);

inline cudaStream_t as_cuda(orStream_t s) {
  return reinterpret_cast<cudaStream_t>(s);
}

#define MCPU_CUDA_TRY(expr, what)                         \
  do {                                                    \
    cudaError_t _st = (expr);                             \
    if (_st != cudaSuccess) return ::mcpu::from_cuda(_st, what); \
  } while (0)

#define MCPU_ARG_CHECK(cond, ...)                         \
  do {                                                    \
    if (!(cond)) {                                        \
      ::mcpu::set_last_error(__VA_ARGS__);                \
      return orErrorInvalidValue;                         \
    }                                                     \
  } while (0)

__device__ __forceinline__ float bf16_bits_to_float(uint16_t h) {
  return __uint_as_float(static_cast<uint32_t>(h) << 16);
}

// Round-to-nearest-even fp32 -> bf16 bits (finite values; NaN kept quiet).
__device__ __forceinline__ uint16_t float_to_bf16_bits(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

// Two roundings in one conversion instruction: bits of bf16(lo) in the low
// half, bf16(hi) in the high half.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

__device__ __forceinline__ float round_bf16(float f) {
  return bf16_bits_to_float(float_to_bf16_bits(f));
}

}  // namespace mcpu
