// silu_and_mul and rms_norm: single-pass HBM-bound kernels for sm_100a.
//
// silu_and_mul: out[t, j] = bf16( bf16(silu(a)) * b ), a = x[t, j],
//   b = x[t, d + j].  vLLM's SiluAndMul.forward_native
//   (vllm/model_executor/layers/activation.py:135-139) executed on the
//   reference's mcpu device: the raw silu loop a / (1.0f + std::exp(-a))
//   (csrc/aten/ops/unary_out.cpp:50-51) rounds to bf16, then aten mul
//   (binary_out.cpp:544-560) multiplies in fp32 and rounds to bf16.  The
//   product of two bf16 values is exact in fp32, so only the silu -> bf16
//   rounding can depend on how exp is evaluated.  The kernel evaluates silu
//   with ex2.approx/rcp.approx and, when the fp32 result lies within its
//   error bound of a bf16 rounding midpoint (about 1e-4 of elements) or |a|
//   is large, re-evaluates it with the correctly rounded exp of expf_cr.h;
//   the bf16 result therefore equals the reference formula's.
//
// rms_norm: vLLM rms_norm native (vllm/ir/ops/layernorm.py:14-21) on bf16:
//   var = mean(float(x)^2); y = bf16(float(x) * (1 / sqrt(var + eps)));
//   out = bf16(float(y) * float(w)).  One CTA per row keeps the row in
//   registers, so x is read once and out written once; the sum of squares is
//   accumulated in fp64 so the mean is the correctly rounded fp32 value
//   (independent of summation order).
#include <math.h>

#include "common.cuh"
#include "expf_cr.h"

namespace mcpu {
namespace bw {

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

__device__ __noinline__ float silu_exact(float a) { return crexp::silu_cr(a); }

// bf16(silu(a)) as the reference computes it.
__device__ __forceinline__ float silu_bf16(float a) {
  const float aa = fabsf(a);
  if (aa <= 60.0f) {
    const float e = ex2_approx(__fmul_rn(a, -1.4426950408889634f));
    const float s = __fmul_rn(a, rcp_approx(__fadd_rn(1.0f, e)));
    // error of s against the reference value, in fp32 ulps of s:
    // <= 12 + 2|a|; stay clear of the bf16 midpoint (low half == 0x8000)
    // with a 2x margin on that bound
    const int low = static_cast<int>(__float_as_uint(s) & 0xFFFFu) - 0x8000;
    const int window = 32 + 4 * static_cast<int>(aa + 1.0f);
    if (abs(low) > window && s != 0.0f) return round_bf16(s);
  }
  return round_bf16(silu_exact(a));
}

__device__ __forceinline__ uint32_t silu_mul_pair(uint32_t a2, uint32_t b2) {
  const float a0 = __uint_as_float(a2 << 16), a1 = __uint_as_float(a2 & 0xFFFF0000u);
  const float b0 = __uint_as_float(b2 << 16), b1 = __uint_as_float(b2 & 0xFFFF0000u);
  const uint32_t o0 = float_to_bf16_bits(__fmul_rn(silu_bf16(a0), b0));
  const uint32_t o1 = float_to_bf16_bits(__fmul_rn(silu_bf16(a1), b1));
  return o0 | (o1 << 16);
}

__device__ __forceinline__ uint4 ldg_stream(const uint4* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ void stg_stream(uint4* p, uint4 v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

// 8 outputs (16 bytes) per vector; d % 8 == 0 and 16-byte aligned rows.
__global__ void __launch_bounds__(256) silu_and_mul_vec_kernel(const uint4* __restrict__ x,
                                                              uint4* __restrict__ out,
                                                              long long T, long long dv) {
  const long long total = T * dv;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += 2 * stride) {
    const long long i2 = i + stride;
    const long long t = i / dv, j = i - t * dv;
    const uint4 a = ldg_stream(x + t * 2 * dv + j);
    const uint4 b = ldg_stream(x + t * 2 * dv + dv + j);
    uint4 a2 = make_uint4(0, 0, 0, 0), b2 = a2;
    long long t2 = 0, j2 = 0;
    if (i2 < total) {
      t2 = i2 / dv;
      j2 = i2 - t2 * dv;
      a2 = ldg_stream(x + t2 * 2 * dv + j2);
      b2 = ldg_stream(x + t2 * 2 * dv + dv + j2);
    }
    uint4 o;
    o.x = silu_mul_pair(a.x, b.x);
    o.y = silu_mul_pair(a.y, b.y);
    o.z = silu_mul_pair(a.z, b.z);
    o.w = silu_mul_pair(a.w, b.w);
    stg_stream(out + t * dv + j, o);
    if (i2 < total) {
      uint4 o2;
      o2.x = silu_mul_pair(a2.x, b2.x);
      o2.y = silu_mul_pair(a2.y, b2.y);
      o2.z = silu_mul_pair(a2.z, b2.z);
      o2.w = silu_mul_pair(a2.w, b2.w);
      stg_stream(out + t2 * dv + j2, o2);
    }
  }
}

__global__ void silu_and_mul_scalar_kernel(const uint16_t* __restrict__ x, uint16_t* __restrict__ out,
                                           long long T, long long d) {
  const long long total = T * d;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long t = i / d, j = i - t * d;
    const float a = bf16_bits_to_float(x[t * 2 * d + j]);
    const float b = bf16_bits_to_float(x[t * 2 * d + d + j]);
    out[i] = float_to_bf16_bits(__fmul_rn(silu_bf16(a), b));
  }
}

// ------------------------------------------------------------------ rms_norm
constexpr int kRmsThreads = 256;
constexpr int kRmsMaxVec = 8;  // vectors of 8 bf16 per thread: H <= 16384

__device__ __forceinline__ double block_sum(double v, double* smem) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, off);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) smem[warp] = v;
  __syncthreads();
  double r = 0.0;
  const int nw = blockDim.x >> 5;
  for (int i = 0; i < nw; ++i) r += smem[i];  // same order in every thread
  return r;
}

__device__ __forceinline__ float normed(float v, float r, float w) {
  const float y = round_bf16(__fmul_rn(v, r));
  return __fmul_rn(y, w);
}

__global__ void __launch_bounds__(kRmsThreads) rms_norm_vec_kernel(
    const uint4* __restrict__ x, const uint4* __restrict__ w, uint4* __restrict__ out, int hv,
    double count, float eps) {
  __shared__ double red[kRmsThreads / 32];
  const long long row = blockIdx.x;
  const uint4* xr = x + row * hv;
  uint4 v[kRmsMaxVec];
  double acc = 0.0;
#pragma unroll
  for (int k = 0; k < kRmsMaxVec; ++k) {
    const int c = threadIdx.x + k * kRmsThreads;
    v[k] = c < hv ? ldg_stream(xr + c) : make_uint4(0, 0, 0, 0);
    const uint32_t q[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float lo = __uint_as_float(q[e] << 16), hi = __uint_as_float(q[e] & 0xFFFF0000u);
      acc += static_cast<double>(__fmul_rn(lo, lo));
      acc += static_cast<double>(__fmul_rn(hi, hi));
    }
  }
  const double total = block_sum(acc, red);
  const float var = static_cast<float>(total / count);
  const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
  uint4* orow = out + row * hv;
#pragma unroll
  for (int k = 0; k < kRmsMaxVec; ++k) {
    const int c = threadIdx.x + k * kRmsThreads;
    if (c < hv) {
      const uint4 wv = __ldg(w + c);
      const uint32_t q[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
      const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
      uint32_t o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float lo = normed(__uint_as_float(q[e] << 16), r, __uint_as_float(ww[e] << 16));
        const float hi = normed(__uint_as_float(q[e] & 0xFFFF0000u), r,
                                __uint_as_float(ww[e] & 0xFFFF0000u));
        o[e] = float_to_bf16_bits(lo) | (static_cast<uint32_t>(float_to_bf16_bits(hi)) << 16);
      }
      stg_stream(orow + c, make_uint4(o[0], o[1], o[2], o[3]));
    }
  }
}

// Any H, any alignment: two passes over the row (the second pass re-reads x).
__global__ void __launch_bounds__(kRmsThreads) rms_norm_scalar_kernel(
    const uint16_t* __restrict__ x, const uint16_t* __restrict__ w, uint16_t* __restrict__ out,
    long long H, double count, float eps) {
  __shared__ double red[kRmsThreads / 32];
  const long long row = blockIdx.x;
  const uint16_t* xr = x + row * H;
  double acc = 0.0;
  for (long long j = threadIdx.x; j < H; j += blockDim.x) {
    const float v = bf16_bits_to_float(xr[j]);
    acc += static_cast<double>(__fmul_rn(v, v));
  }
  const double total = block_sum(acc, red);
  const float var = static_cast<float>(total / count);
  const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
  for (long long j = threadIdx.x; j < H; j += blockDim.x)
    out[row * H + j] = float_to_bf16_bits(normed(bf16_bits_to_float(xr[j]), r, bf16_bits_to_float(w[j])));
}

static int sm_count() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

}  // namespace bw
}  // namespace mcpu

using namespace mcpu;

extern "C" orError_t mcpu_silu_and_mul(void* out, const void* x, int64_t num_tokens, int64_t d,
                                       int dtype, orStream_t stream) {
  MCPU_ARG_CHECK(dtype == MCPU_BFLOAT16, "silu_and_mul: only bfloat16 is supported (dtype code %d)",
                 dtype);
  MCPU_ARG_CHECK(num_tokens >= 0 && d >= 0, "silu_and_mul: negative size");
  if (num_tokens == 0 || d == 0) return orSuccess;
  MCPU_ARG_CHECK(out && x, "silu_and_mul: NULL tensor pointer");
  cudaStream_t st = as_cuda(stream);
  const bool vec = d % 8 == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(out) % 16 == 0;
  const int blocks = bw::sm_count() * 8;
  if (vec) {
    bw::silu_and_mul_vec_kernel<<<blocks, 256, 0, st>>>(static_cast<const uint4*>(x),
                                                         static_cast<uint4*>(out), num_tokens, d / 8);
  } else {
    bw::silu_and_mul_scalar_kernel<<<blocks, 256, 0, st>>>(static_cast<const uint16_t*>(x),
                                                           static_cast<uint16_t*>(out), num_tokens, d);
  }
  return from_cuda(cudaGetLastError(), "silu_and_mul launch");
}

extern "C" orError_t mcpu_rms_norm(void* out, const void* x, const void* weight, int64_t num_tokens,
                                   int64_t hidden, float eps, int dtype, orStream_t stream) {
  MCPU_ARG_CHECK(dtype == MCPU_BFLOAT16, "rms_norm: only bfloat16 is supported (dtype code %d)", dtype);
  MCPU_ARG_CHECK(num_tokens >= 0 && hidden > 0, "rms_norm: bad size (tokens %lld, hidden %lld)",
                 (long long)num_tokens, (long long)hidden);
  MCPU_ARG_CHECK(num_tokens <= 0x7FFFFFFFLL, "rms_norm: too many rows");
  if (num_tokens == 0) return orSuccess;
  MCPU_ARG_CHECK(out && x && weight, "rms_norm: NULL tensor pointer");
  cudaStream_t st = as_cuda(stream);
  const bool vec = hidden % 8 == 0 && hidden / 8 <= bw::kRmsThreads * bw::kRmsMaxVec &&
                   reinterpret_cast<uintptr_t>(x) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(out) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(weight) % 16 == 0;
  const double count = static_cast<double>(hidden);
  if (vec) {
    bw::rms_norm_vec_kernel<<<static_cast<unsigned>(num_tokens), bw::kRmsThreads, 0, st>>>(
        static_cast<const uint4*>(x), static_cast<const uint4*>(weight), static_cast<uint4*>(out),
        static_cast<int>(hidden / 8), count, eps);
  } else {
    bw::rms_norm_scalar_kernel<<<static_cast<unsigned>(num_tokens), bw::kRmsThreads, 0, st>>>(
        static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(weight),
        static_cast<uint16_t*>(out), hidden, count, eps);
  }
  return from_cuda(cudaGetLastError(), "rms_norm launch");
}
