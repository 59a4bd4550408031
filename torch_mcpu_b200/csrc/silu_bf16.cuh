// silu in fp32 accurate enough to round to the reference's bf16 value, for
// the bf16 paths (silu_and_mul, the GEMM's SwiGLU epilogue).  The reference
// computes silu as g / (1.0f + expf(-g)) in fp32 (csrc/aten/ops/
// unary_out.cpp:50-51) and rounds to bf16.
#pragma once

#include "common.cuh"
#include "expf_cr.h"

namespace mcpu {

// The reference formula with exp correctly rounded, out of line: the rare
// path, kept out of the callers' registers.
__device__ __noinline__ inline float silu_cr_call(float a) { return crexp::silu_cr(a); }

// Fast form (ex2.approx, rcp.approx) when its result is clear of a bf16
// rounding midpoint, else the reference formula.  The fast form's error
// against the reference value is at most 12 + 2|a| fp32 ulps of s; the test
// keeps twice that away from the midpoint (low half == 0x8000): a fixed 56
// ulps for |a| <= 8 (every N(0,1) activation), 32 + 4 (|a| + 1) bounded by
// 36 + (8 << k) for |a| in [2^k, 2^(k+1)) up to 60.
__device__ __forceinline__ float silu_for_bf16(float a) {
  float e, r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(__fmul_rn(a, -1.4426950408889634f)));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(__fadd_rn(1.0f, e)));
  const float s = __fmul_rn(a, r);
  const int low = static_cast<int>(__float_as_uint(s) & 0xFFFFu) - 0x8000;
  const float aa = fabsf(a);
  if (aa <= 8.0f) {
    if (abs(low) > 56) return s;
  } else if (aa <= 60.0f) {
    const int ea = static_cast<int>((__float_as_uint(a) >> 23) & 0xFFu) - 127;
    if (abs(low) > 36 + (8 << ea)) return s;
  }
  return silu_cr_call(a);
}

// The fast form alone, with *exact set when its bf16 rounding is not
// certain (|a| > 8, or within 56 ulps of a midpoint): no branch, so a
// vector of elements runs straight and the rare fix-ups follow.
__device__ __forceinline__ float silu_fast_checked(float a, bool* exact) {
  float e, r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(__fmul_rn(a, -1.4426950408889634f)));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(__fadd_rn(1.0f, e)));
  const float s = __fmul_rn(a, r);
  const int low = static_cast<int>(__float_as_uint(s) & 0xFFFFu) - 0x8000;
  *exact = !(fabsf(a) <= 8.0f) || abs(low) <= 56;
  return s;
}

}  // namespace mcpu
