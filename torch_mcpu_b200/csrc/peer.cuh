// System-scope memory operations for kernels that exchange data with the
// other GPUs of the box through CUDA IPC mappings (NVLink / NVSwitch peer
// memory): plain vector stores to a peer, release/acquire counters, and a
// bounded wait that gives up after a fixed wall time instead of hanging.
#pragma once

#include <stdint.h>

namespace mcpu {
namespace peer {

// Longest a kernel waits for another GPU before it records an error and
// leaves: far above any legitimate skew between the ranks of one step.
constexpr unsigned long long kWaitNs = 2000000000ull;
// Second bound on the same wait, in polls, in case the timer does not move.
constexpr uint32_t kWaitPolls = 1u << 26;

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// 16-byte store to global memory (local or a peer's mapping).
__device__ __forceinline__ void st_v4(void* p, const uint4& v) {
  asm volatile("st.global.v4.b32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

// 16-byte load that skips L1 (the data was written by other GPUs during
// this kernel).
__device__ __forceinline__ uint4 ld_cg_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

// Orders this thread's earlier stores (to any GPU) before its later ones.
__device__ __forceinline__ void fence_sys() {
  asm volatile("fence.acq_rel.sys;" ::: "memory");
}

__device__ __forceinline__ void red_add_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Waits until *p >= target.  False when neither bound let it finish.
__device__ __forceinline__ bool wait_geq_sys(const uint32_t* p, uint32_t target) {
  const unsigned long long t0 = globaltimer();
  for (uint32_t i = 0; i < kWaitPolls; ++i) {
    if (ld_acquire_sys(p) >= target) return true;
    if ((i & 31u) == 31u && globaltimer() - t0 > kWaitNs) return false;
    __nanosleep(32);
  }
  return false;
}

}  // namespace peer
}  // namespace mcpu
