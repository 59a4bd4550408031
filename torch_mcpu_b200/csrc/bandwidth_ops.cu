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
#include "silu_bf16.cuh"
#include "sm100.cuh"

namespace mcpu {
namespace bw {


// out = bf16(bf16(silu(a)) * b) for 8 bf16 pairs (a and b vectors): the
// fast silu of all eight, then the few elements whose rounding is not
// certain redone with the reference formula, then two roundings per
// conversion instruction.
__device__ __forceinline__ uint4 silu_mul_vec(uint4 av, uint4 bv) {
  const uint32_t aw[4] = {av.x, av.y, av.z, av.w};
  const uint32_t bw[4] = {bv.x, bv.y, bv.z, bv.w};
  float a[8], s[8];
  uint32_t redo = 0;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    a[2 * q] = __uint_as_float(aw[q] << 16);
    a[2 * q + 1] = __uint_as_float(aw[q] & 0xFFFF0000u);
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    bool ex;
    s[j] = silu_fast_checked(a[j], &ex);
    redo |= ex ? (1u << j) : 0u;
  }
  if (redo) {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (redo & (1u << j)) s[j] = silu_cr_call(a[j]);
  }
  uint32_t o[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint32_t s2 = pack_bf16x2(s[2 * q], s[2 * q + 1]);
    o[q] = pack_bf16x2(__fmul_rn(__uint_as_float(s2 << 16), __uint_as_float(bw[q] << 16)),
                       __fmul_rn(__uint_as_float(s2 & 0xFFFF0000u), __uint_as_float(bw[q] & 0xFFFF0000u)));
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
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
// CTAs loop over rows, so no index division; each thread keeps three
// vector pairs in flight.
__global__ void __launch_bounds__(256) silu_and_mul_rows_kernel(const uint4* __restrict__ x,
                                                               uint4* __restrict__ out,
                                                               long long T, int dv) {
  for (long long t = blockIdx.x; t < T; t += gridDim.x) {
    const uint4* a = x + t * 2 * dv;
    const uint4* b = a + dv;
    uint4* o = out + t * dv;
    int j = threadIdx.x;
    for (; j + 2 * 256 < dv; j += 3 * 256) {
      uint4 av[3], bv[3];
#pragma unroll
      for (int u = 0; u < 3; ++u) {
        av[u] = ldg_stream(a + j + u * 256);
        bv[u] = ldg_stream(b + j + u * 256);
      }
#pragma unroll
      for (int u = 0; u < 3; ++u) stg_stream(o + j + u * 256, silu_mul_vec(av[u], bv[u]));
    }
    for (; j < dv; j += 256) {
      stg_stream(o + j, silu_mul_vec(ldg_stream(a + j), ldg_stream(b + j)));
    }
  }
}

// Narrow rows (fewer than 256 vectors): one flat index space.
__global__ void __launch_bounds__(256) silu_and_mul_flat_kernel(const uint4* __restrict__ x,
                                                               uint4* __restrict__ out,
                                                               long long T, long long dv) {
  const long long total = T * dv;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long t = i / dv, j = i - t * dv;
    stg_stream(out + i, silu_mul_vec(ldg_stream(x + t * 2 * dv + j), ldg_stream(x + t * 2 * dv + dv + j)));
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
    out[i] = float_to_bf16_bits(__fmul_rn(round_bf16(silu_for_bf16(a)), b));
  }
}

// ------------------------------------------------------------------ rms_norm
constexpr int kRmsThreads = 256;

__device__ int g_bw_error = 0;

// Sum over the CTA in a fixed order (identical in every thread).  The
// barrier also ORs `fail` over the CTA into *any_fail.
__device__ __forceinline__ double block_sum(double v, double* smem, bool fail = false,
                                           bool* any_fail = nullptr) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, off);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) smem[warp] = v;
  const int f = __syncthreads_or(fail ? 1 : 0);
  if (any_fail) *any_fail = f != 0;
  double r = 0.0;
  const int nw = blockDim.x >> 5;
  for (int i = 0; i < nw; ++i) r += smem[i];
  return r;
}

// x * x of a bf16 value (exact in fp32 for normal products), in double.
__device__ __forceinline__ double square_as_double(float v) {
  return static_cast<double>(__fmul_rn(v, v));
}

__device__ __forceinline__ float normed(float v, float r, float w) {
  const float y = round_bf16(__fmul_rn(v, r));
  return __fmul_rn(y, w);
}

// Persistent CTAs; rows stream through a ring of `stages` shared-memory row
// buffers filled by bulk copies (one mbarrier per buffer), so the next rows
// are in flight while this one is reduced.  Each thread owns the vectors
// c = threadIdx.x + k * 256 of a row and of the weight.
// Rows are 16-byte multiples (H % 8 == 0) and 16-byte aligned.
template <int NV>
__global__ void __launch_bounds__(kRmsThreads, NV <= 4 ? 4 : 1) rms_norm_ring_kernel(
    const uint8_t* __restrict__ x, const uint4* __restrict__ w, uint4* __restrict__ out, int hv,
    long long T, int stages, double count, float eps) {
  extern __shared__ __align__(128) uint8_t ring[];
  const int row_bytes = hv * 16;
  const int slot = (row_bytes + 127) & ~127;
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + stages * slot);
  double* red = reinterpret_cast<double*>(full + stages);  // [2][kRmsThreads / 32]
  int* abort_flag = reinterpret_cast<int*>(red + 2 * (kRmsThreads / 32));

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) sm100::mbar_init(&full[s], 1);
    *abort_flag = 0;
    sm100::fence_barrier_init();
    for (int s = 0; s < stages; ++s) {
      const long long row = blockIdx.x + static_cast<long long>(s) * gridDim.x;
      if (row < T) {
        sm100::mbar_arrive_expect_tx(&full[s], row_bytes);
        sm100::bulk_load(ring + s * slot, x + row * row_bytes, row_bytes, &full[s]);
      }
    }
  }
  __syncthreads();

  int i = 0;
  for (;; ++i) {
    const long long row = blockIdx.x + static_cast<long long>(i) * gridDim.x;
    if (row >= T) break;
    const int st = i % stages;
    const bool ok = sm100::mbar_wait(&full[st], (i / stages) & 1, abort_flag);
    const uint4* src = reinterpret_cast<const uint4*>(ring + st * slot);
    uint4 v[NV];
    double acc = 0.0;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int c = threadIdx.x + k * kRmsThreads;
      v[k] = (ok && c < hv) ? src[c] : make_uint4(0, 0, 0, 0);
      const uint32_t q[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        acc += square_as_double(__uint_as_float(q[e] << 16));
        acc += square_as_double(__uint_as_float(q[e] & 0xFFFF0000u));
      }
    }
    // after this barrier every thread has read buffer st: refill it (or
    // leave together when any thread's wait gave up)
    bool failed = false;
    const double total = block_sum(acc, red + (i & 1) * (kRmsThreads / 32), !ok, &failed);
    if (failed) {
      if (threadIdx.x == 0) *abort_flag = 1;
      break;
    }
    if (threadIdx.x == 0) {
      const long long nrow = row + static_cast<long long>(stages) * gridDim.x;
      if (nrow < T) {
        sm100::mbar_arrive_expect_tx(&full[st], row_bytes);
        sm100::bulk_load(ring + st * slot, x + nrow * row_bytes, row_bytes, &full[st]);
      }
    }
    const float var = static_cast<float>(total / count);
    const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
    uint4* orow = out + row * hv;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int c = threadIdx.x + k * kRmsThreads;
      if (c < hv) {
        const uint4 wv = __ldg(w + c);  // 2H bytes, L1-resident across rows
        const uint32_t q[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
        const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          // y = bf16(x * r) for both halves in one conversion, then bf16(y * w)
          const uint32_t y2 = pack_bf16x2(__fmul_rn(__uint_as_float(q[e] << 16), r),
                                          __fmul_rn(__uint_as_float(q[e] & 0xFFFF0000u), r));
          o[e] = pack_bf16x2(__fmul_rn(__uint_as_float(y2 << 16), __uint_as_float(ww[e] << 16)),
                             __fmul_rn(__uint_as_float(y2 & 0xFFFF0000u), __uint_as_float(ww[e] & 0xFFFF0000u)));
        }
        stg_stream(orow + c, make_uint4(o[0], o[1], o[2], o[3]));
      }
    }
  }
  if (threadIdx.x == 0 && *abort_flag) {
    // a wait ran out: record it, then let the copies this CTA issued land
    atomicExch(&g_bw_error, 1);
    for (int j = i; j < i + stages; ++j) {
      if (blockIdx.x + static_cast<long long>(j) * gridDim.x >= T) break;
      for (uint32_t n = 0; n < sm100::kSpinLimit && !sm100::mbar_try_wait(&full[j % stages], (j / stages) & 1);
           ++n) {
      }
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
    acc += square_as_double(v);
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

// Ring depth: up to 4 row buffers within 48 KB of shared memory (at least 2).
template <int NV>
static cudaError_t launch_rms_ring(void* out, const void* x, const void* w, int hv, long long T,
                                   double count, float eps, cudaStream_t st) {
  auto kern = rms_norm_ring_kernel<NV>;
  const int slot = (hv * 16 + 127) & ~127;
  int stages = (48 * 1024) / slot;
  stages = stages < 2 ? 2 : (stages > 4 ? 4 : stages);
  const int smem = stages * slot + stages * 8 + 2 * (kRmsThreads / 32) * 8 + 16;
  if (smem > 48 * 1024) {
    cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), smem);
    if (e != cudaSuccess) return e;
  }
  int per_sm = 1;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kRmsThreads, smem);
  if (per_sm < 1) per_sm = 1;
  const long long cap = static_cast<long long>(sm_count()) * per_sm;
  const int grid = static_cast<int>(T < cap ? T : cap);
  kern<<<grid, kRmsThreads, smem, st>>>(static_cast<const uint8_t*>(x), static_cast<const uint4*>(w),
                                        static_cast<uint4*>(out), hv, T, stages, count, eps);
  return cudaGetLastError();
}

orError_t read_error(int* flag, bool reset) {
  MCPU_CUDA_TRY(cudaMemcpyFromSymbol(flag, g_bw_error, sizeof(int)), "rms_norm error flag");
  if (reset) {
    const int zero = 0;
    MCPU_CUDA_TRY(cudaMemcpyToSymbol(g_bw_error, &zero, sizeof(int)), "rms_norm error flag reset");
  }
  return orSuccess;
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
  if (vec && d / 8 >= 256 && d / 8 <= 0x7FFFFFFF) {
    const long long grid = num_tokens < blocks ? num_tokens : blocks;
    bw::silu_and_mul_rows_kernel<<<static_cast<unsigned>(grid), 256, 0, st>>>(
        static_cast<const uint4*>(x), static_cast<uint4*>(out), num_tokens, static_cast<int>(d / 8));
  } else if (vec) {
    bw::silu_and_mul_flat_kernel<<<blocks, 256, 0, st>>>(static_cast<const uint4*>(x),
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
  const int hv = static_cast<int>(hidden / 8);
  const bool ring = hidden % 8 == 0 && hv <= bw::kRmsThreads * 8 &&
                    reinterpret_cast<uintptr_t>(x) % 16 == 0 &&
                    reinterpret_cast<uintptr_t>(out) % 16 == 0 &&
                    reinterpret_cast<uintptr_t>(weight) % 16 == 0;
  const double count = static_cast<double>(hidden);
  if (ring) {
    const int nv = (hv + bw::kRmsThreads - 1) / bw::kRmsThreads;
    cudaError_t e;
    if (nv <= 1) e = bw::launch_rms_ring<1>(out, x, weight, hv, num_tokens, count, eps, st);
    else if (nv <= 2) e = bw::launch_rms_ring<2>(out, x, weight, hv, num_tokens, count, eps, st);
    else if (nv <= 4) e = bw::launch_rms_ring<4>(out, x, weight, hv, num_tokens, count, eps, st);
    else e = bw::launch_rms_ring<8>(out, x, weight, hv, num_tokens, count, eps, st);
    return from_cuda(e, "rms_norm launch");
  } else {
    bw::rms_norm_scalar_kernel<<<static_cast<unsigned>(num_tokens), bw::kRmsThreads, 0, st>>>(
        static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(weight),
        static_cast<uint16_t*>(out), hidden, count, eps);
  }
  return from_cuda(cudaGetLastError(), "rms_norm launch");
}
