// Device helpers shared by the grouped_topk kernels (grouped_topk.cu,
// grouped_topk_tma.cu).
#pragma once

#include <math.h>

#include "common.cuh"
#include "expf_cr.h"

namespace mcpu {
namespace router {

constexpr int kThreads = 256;

__device__ __forceinline__ float ex2_approx(float y) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(y));
  return r;
}

__device__ __forceinline__ float rcp_approx(float y) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(y));
  return r;
}

// Fast sigmoid used only for ranking; |error| < 2^-21 absolute: the exponent
// argument carries |x| 2^-24 relative error, ex2.approx about 2^-22, the sum
// and the approximate reciprocal one rounding each, and s(1-s) <= 1/4 damps
// the exp error.
__device__ __forceinline__ float sigmoid_fast(float x) {
  const float e = ex2_approx(__fmul_rn(x, -1.4426950408889634f));
  return rcp_approx(__fadd_rn(1.0f, e));
}

// The reference formula 1.0f / (1.0f + expf(-x)) with exp correctly
// rounded (fp32 arithmetic only, see expf_cr.h).
__device__ __forceinline__ float sigmoid_exact(float x) { return crexp::sigmoid_cr(x); }

// Out-of-line copy for the rare exact paths: keeps their code and registers
// out of the unrolled fast paths.
__device__ __noinline__ float sigmoid_exact_call(float x) { return sigmoid_exact(x); }

__device__ __forceinline__ float fast_key(float x, float b) {
  return __fadd_rn(sigmoid_fast(x), b);
}

__device__ __forceinline__ uint32_t orderable(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Keys packed so that an unsigned compare ranks by value, then by lower
// index.  0 means "no element".
struct Pack32 {
  using T = uint32_t;
  static __device__ __forceinline__ T pack(float f, int idx, uint32_t mask) {
    return (orderable(f) & ~mask) | (mask - static_cast<uint32_t>(idx));
  }
  static __device__ __forceinline__ int index(T k, uint32_t mask) {
    return static_cast<int>(mask - (k & mask));
  }
};

struct Pack64 {
  using T = unsigned long long;
  static __device__ __forceinline__ T pack(float f, int idx, uint32_t) {
    return (static_cast<T>(orderable(f)) << 32) |
           static_cast<T>(0xFFFFFFFFu - static_cast<uint32_t>(idx));
  }
  static __device__ __forceinline__ int index(T k, uint32_t) {
    return static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(k));
  }
};

template <typename K>
__device__ __forceinline__ K kmax(K a, K b) { return a > b ? a : b; }
template <typename K>
__device__ __forceinline__ K kmin(K a, K b) { return a > b ? b : a; }

template <typename K, int N>
__device__ __forceinline__ void bitonic_sort_desc(K (&a)[N]) {
#pragma unroll
  for (int k = 2; k <= N; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
#pragma unroll
      for (int i = 0; i < N; ++i) {
        const int l = i ^ j;
        if (l > i) {
          const K x = a[i], y = a[l];
          const K hi = kmax(x, y), lo = kmin(x, y);
          if ((i & k) == 0) {
            a[i] = hi;
            a[l] = lo;
          } else {
            a[i] = lo;
            a[l] = hi;
          }
        }
      }
    }
  }
}

template <typename K, int N>
__device__ __forceinline__ void bitonic_merge_desc(K (&a)[N]) {
#pragma unroll
  for (int j = N >> 1; j > 0; j >>= 1) {
#pragma unroll
    for (int i = 0; i < N; ++i) {
      const int l = i ^ j;
      if (l > i) {
        const K x = a[i], y = a[l];
        a[i] = kmax(x, y);
        a[l] = kmin(x, y);
      }
    }
  }
}

// best = the L largest of pk[0..GS_MAX), sorted descending.
template <typename K, int L, int GS_MAX>
__device__ __forceinline__ void local_top(const K (&pk)[GS_MAX], K (&best)[L]) {
  if constexpr (GS_MAX <= L) {
#pragma unroll
    for (int i = 0; i < L; ++i) best[i] = i < GS_MAX ? pk[i] : K(0);
    bitonic_sort_desc(best);
  } else {
#pragma unroll
    for (int i = 0; i < L; ++i) best[i] = pk[i];
    bitonic_sort_desc(best);
#pragma unroll
    for (int c = 1; c < GS_MAX / L; ++c) {
      K t[L];
#pragma unroll
      for (int i = 0; i < L; ++i) t[i] = pk[c * L + i];
      bitonic_sort_desc(t);
#pragma unroll
      for (int i = 0; i < L; ++i) best[i] = kmax(best[i], t[L - 1 - i]);
      bitonic_merge_desc(best);
    }
  }
}

// Butterfly all-merge of the sorted top-L lists of the G lanes of a segment.
template <typename K, int L>
__device__ __forceinline__ void segment_merge(K (&best)[L], unsigned segmask, int G) {
  for (int off = 1; off < G; off <<= 1) {
    K o[L];
#pragma unroll
    for (int i = 0; i < L; ++i) o[i] = __shfl_xor_sync(segmask, best[i], off, G);
#pragma unroll
    for (int i = 0; i < L; ++i) best[i] = kmax(best[i], o[L - 1 - i]);
    bitonic_merge_desc(best);
  }
}

template <typename K, int L>
__device__ __forceinline__ K select_at(const K (&a)[L], int i) {
  K r = 0;
#pragma unroll
  for (int j = 0; j < L; ++j) r = (j == i) ? a[j] : r;
  return r;
}

__device__ __forceinline__ float seg_max(float v, unsigned m, int G) {
  for (int off = 1; off < G; off <<= 1) v = fmaxf(v, __shfl_xor_sync(m, v, off, G));
  return v;
}
__device__ __forceinline__ float seg_min(float v, unsigned m, int G) {
  for (int off = 1; off < G; off <<= 1) v = fminf(v, __shfl_xor_sync(m, v, off, G));
  return v;
}
__device__ __forceinline__ float seg_sum(float v, unsigned m, int G) {
  for (int off = 1; off < G; off <<= 1) v = __fadd_rn(v, __shfl_xor_sync(m, v, off, G));
  return v;
}
template <typename K>
__device__ __forceinline__ K seg_kmax(K v, unsigned m, int G) {
  for (int off = 1; off < G; off <<= 1) v = kmax(v, __shfl_xor_sync(m, v, off, G));
  return v;
}

struct Params {
  const void* gating;
  const float* bias;
  float* w_out;
  int32_t* id_out;
  long long T;
  int E, G, GS, TG, K;
  int renorm;
  float scale;
  int scoring;   // mcpuScoring
  uint32_t idx_mask;  // (1 << idx_bits) - 1 for the 32-bit keys
  float idx_quantum;  // 2^(idx_bits - 23): relative truncation of a 32-bit key
};

template <typename InT>
__device__ __forceinline__ float load_one(const InT* p);
template <>
__device__ __forceinline__ float load_one<float>(const float* p) { return __ldg(p); }
template <>
__device__ __forceinline__ float load_one<__nv_bfloat16>(const __nv_bfloat16* p) {
  return bf16_bits_to_float(__ldg(reinterpret_cast<const unsigned short*>(p)));
}


__device__ __forceinline__ float sigmoid_accurate(float x) {
  return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x)));
}

}  // namespace router
}  // namespace mcpu
