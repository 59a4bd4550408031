// Device-side tensor plumbing of the mcpu device on B200: stream-ordered
// allocation, strided copy with dtype conversion, fill, and the elementwise
// ops the reference registers for its raw loops (sigmoid, silu, mul).
//
// Reference counterparts (kzwrime/torch_mcpu):
//   allocation   csrc/runtime/DeviceCachingAllocator.cpp (caching allocator,
//                record_stream through events) -> cudaMallocAsync/FreeAsync
//                on a device memory pool that keeps freed memory cached
//   copy         csrc/aten/native/Minimal.cpp:393-484 (_copy_from)
//   fill/zero    csrc/aten/ops/fill.cpp:12-44, unary_out.cpp:239-267
//   sigmoid/silu csrc/aten/ops/unary_out.cpp:46-51 raw loops, computed here
//                with exp correctly rounded (the fp32 result of the raw
//                formula; bf16 results are rounded from it)
//   mul          csrc/aten/ops/binary_out.cpp:544-560
#include <math.h>

#include <mutex>

#include "common.cuh"
#include "expf_cr.h"

namespace mcpu {
namespace tensor {

constexpr int kMaxDims = 8;

struct Strided {
  int ndim;
  long long sizes[kMaxDims];
  long long src[kMaxDims];  // element strides
  long long dst[kMaxDims];
};

template <int DT>
struct Ty;
template <> struct Ty<MCPU_FLOAT32> { using T = float; static constexpr bool fp = true; };
template <> struct Ty<MCPU_BFLOAT16> { using T = uint16_t; static constexpr bool fp = true; };
template <> struct Ty<MCPU_FLOAT16> { using T = __half; static constexpr bool fp = true; };
template <> struct Ty<MCPU_INT32> { using T = int32_t; static constexpr bool fp = false; };
template <> struct Ty<MCPU_INT64> { using T = long long; static constexpr bool fp = false; };
template <> struct Ty<MCPU_UINT8> { using T = uint8_t; static constexpr bool fp = false; };
template <> struct Ty<MCPU_BOOL> { using T = uint8_t; static constexpr bool fp = false; };
template <> struct Ty<MCPU_FLOAT64> { using T = double; static constexpr bool fp = true; };
template <> struct Ty<MCPU_INT8> { using T = int8_t; static constexpr bool fp = false; };
template <> struct Ty<MCPU_INT16> { using T = int16_t; static constexpr bool fp = false; };

// Values travel as double (floating types) or long long (integer types).
struct Val {
  double d;
  long long i;
  bool is_fp;
};

template <int DT>
__device__ __forceinline__ Val load(const void* p, long long off) {
  using T = typename Ty<DT>::T;
  const T v = static_cast<const T*>(p)[off];
  Val r;
  r.is_fp = Ty<DT>::fp;
  if constexpr (DT == MCPU_BFLOAT16) {
    r.d = static_cast<double>(bf16_bits_to_float(v));
  } else if constexpr (DT == MCPU_FLOAT16) {
    r.d = static_cast<double>(__half2float(v));
  } else if constexpr (Ty<DT>::fp) {
    r.d = static_cast<double>(v);
  } else if constexpr (DT == MCPU_BOOL) {
    r.i = v != 0;
  } else {
    r.i = static_cast<long long>(v);
  }
  if (r.is_fp) r.i = 0; else r.d = 0.0;
  return r;
}

template <int DT>
__device__ __forceinline__ void store(void* p, long long off, Val v) {
  using T = typename Ty<DT>::T;
  T* q = static_cast<T*>(p) + off;
  if constexpr (DT == MCPU_BOOL) {
    *q = v.is_fp ? (v.d != 0.0) : (v.i != 0);
  } else if constexpr (DT == MCPU_BFLOAT16) {
    // double -> float -> bf16 (torch converts through fp32)
    *q = float_to_bf16_bits(v.is_fp ? static_cast<float>(v.d) : static_cast<float>(v.i));
  } else if constexpr (DT == MCPU_FLOAT16) {
    *q = __float2half_rn(v.is_fp ? static_cast<float>(v.d) : static_cast<float>(v.i));
  } else if constexpr (DT == MCPU_FLOAT32) {
    *q = v.is_fp ? static_cast<float>(v.d) : static_cast<float>(v.i);
  } else if constexpr (DT == MCPU_FLOAT64) {
    *q = v.is_fp ? v.d : static_cast<double>(v.i);
  } else {
    *q = static_cast<T>(v.is_fp ? static_cast<long long>(v.d) : v.i);  // truncation toward zero
  }
}

__device__ __forceinline__ void offsets(const Strided& s, long long lin, long long* so, long long* dof) {
  long long a = 0, b = 0;
  for (int d = s.ndim - 1; d >= 0; --d) {
    const long long idx = lin % s.sizes[d];
    lin /= s.sizes[d];
    a += idx * s.src[d];
    b += idx * s.dst[d];
  }
  *so = a;
  *dof = b;
}

template <int DT>
constexpr bool is_f32_family() {
  return DT == MCPU_FLOAT32 || DT == MCPU_BFLOAT16 || DT == MCPU_FLOAT16;
}

template <int DT>
__device__ __forceinline__ float load_f(const void* p, long long off) {
  if constexpr (DT == MCPU_FLOAT32) return static_cast<const float*>(p)[off];
  else if constexpr (DT == MCPU_BFLOAT16) return bf16_bits_to_float(static_cast<const uint16_t*>(p)[off]);
  else return __half2float(static_cast<const __half*>(p)[off]);
}

template <int DT>
__device__ __forceinline__ void store_f(void* p, long long off, float v) {
  if constexpr (DT == MCPU_FLOAT32) static_cast<float*>(p)[off] = v;
  else if constexpr (DT == MCPU_BFLOAT16) static_cast<uint16_t*>(p)[off] = float_to_bf16_bits(v);
  else static_cast<__half*>(p)[off] = __float2half_rn(v);
}

template <int SDT, int DDT>
__global__ void copy_kernel(const void* src, void* dst, const Strided s, long long n) {
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    long long so, dof;
    offsets(s, i, &so, &dof);
    if constexpr (is_f32_family<SDT>() && is_f32_family<DDT>()) {
      store_f<DDT>(dst, dof, load_f<SDT>(src, so));  // fp32 <-> bf16 / fp16 without fp64
    } else {
      store<DDT>(dst, dof, load<SDT>(src, so));
    }
  }
}

template <int DDT>
__global__ void fill_kernel(void* dst, const Strided s, long long n, Val v) {
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    long long so, dof;
    offsets(s, i, &so, &dof);
    store<DDT>(dst, dof, v);
  }
}

#define MCPU_DTYPE_CASES(M, ...)    \
  M(MCPU_FLOAT32, __VA_ARGS__)      \
  M(MCPU_BFLOAT16, __VA_ARGS__)     \
  M(MCPU_FLOAT16, __VA_ARGS__)      \
  M(MCPU_INT32, __VA_ARGS__)        \
  M(MCPU_INT64, __VA_ARGS__)        \
  M(MCPU_UINT8, __VA_ARGS__)        \
  M(MCPU_BOOL, __VA_ARGS__)         \
  M(MCPU_FLOAT64, __VA_ARGS__)      \
  M(MCPU_INT8, __VA_ARGS__)         \
  M(MCPU_INT16, __VA_ARGS__)

template <int SDT>
static cudaError_t launch_copy_to(int ddt, const void* src, void* dst, const Strided& s, long long n,
                                  int blocks, cudaStream_t st) {
  switch (ddt) {
#define CASE(D, ...) \
  case D:            \
    copy_kernel<SDT, D><<<blocks, 256, 0, st>>>(src, dst, s, n); \
    return cudaGetLastError();
    MCPU_DTYPE_CASES(CASE)
#undef CASE
  }
  return cudaErrorInvalidValue;
}

static cudaError_t launch_copy(int sdt, int ddt, const void* src, void* dst, const Strided& s, long long n,
                               int blocks, cudaStream_t st) {
  switch (sdt) {
#define CASE(S, ...) \
  case S:            \
    return launch_copy_to<S>(ddt, src, dst, s, n, blocks, st);
    MCPU_DTYPE_CASES(CASE)
#undef CASE
  }
  return cudaErrorInvalidValue;
}

static bool valid_dtype(int dt) { return dt >= MCPU_FLOAT32 && dt <= MCPU_INT16; }

static int grid_for(long long n) {
  long long b = (n + 255) / 256;
  return static_cast<int>(b < 148 * 16 ? (b > 0 ? b : 1) : 148 * 16);
}

// ---------------------------------------------------------------- elementwise

template <int DT>
__global__ void sigmoid_kernel(const void* x, void* out, long long n) {
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float v;
    if constexpr (DT == MCPU_FLOAT32) v = static_cast<const float*>(x)[i];
    else v = bf16_bits_to_float(static_cast<const uint16_t*>(x)[i]);
    const float s = crexp::sigmoid_cr(v);
    if constexpr (DT == MCPU_FLOAT32) static_cast<float*>(out)[i] = s;
    else static_cast<uint16_t*>(out)[i] = float_to_bf16_bits(s);
  }
}

template <int DT>
__global__ void silu_kernel(const void* x, void* out, long long n) {
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float v;
    if constexpr (DT == MCPU_FLOAT32) v = static_cast<const float*>(x)[i];
    else v = bf16_bits_to_float(static_cast<const uint16_t*>(x)[i]);
    const float s = crexp::silu_cr(v);
    if constexpr (DT == MCPU_FLOAT32) static_cast<float*>(out)[i] = s;
    else static_cast<uint16_t*>(out)[i] = float_to_bf16_bits(s);
  }
}

template <int DT>
__global__ void mul_kernel(const void* a, const void* b, void* out, long long n) {
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    if constexpr (DT == MCPU_FLOAT32) {
      static_cast<float*>(out)[i] = __fmul_rn(static_cast<const float*>(a)[i], static_cast<const float*>(b)[i]);
    } else {
      const float p = __fmul_rn(bf16_bits_to_float(static_cast<const uint16_t*>(a)[i]),
                                bf16_bits_to_float(static_cast<const uint16_t*>(b)[i]));
      static_cast<uint16_t*>(out)[i] = float_to_bf16_bits(p);
    }
  }
}

}  // namespace tensor
}  // namespace mcpu

using namespace mcpu;

extern "C" {

orError_t orMallocAsync(void** devPtr, size_t size, orStream_t stream) {
  MCPU_ARG_CHECK(devPtr != nullptr, "orMallocAsync: devPtr is NULL");
  if (size == 0) {
    *devPtr = nullptr;
    return orSuccess;
  }
  // keep freed blocks in the device's pool instead of returning them to the
  // driver at every synchronisation (a caching allocator's behaviour)
  static std::once_flag once[64];
  int dev = 0;
  MCPU_CUDA_TRY(cudaGetDevice(&dev), "orMallocAsync");
  if (dev >= 0 && dev < 64) {
    std::call_once(once[dev], [dev] {
      cudaMemPool_t pool;
      if (cudaDeviceGetDefaultMemPool(&pool, dev) == cudaSuccess) {
        unsigned long long thr = ~0ull;
        cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thr);
      }
    });
  }
  return from_cuda(cudaMallocAsync(devPtr, size, as_cuda(stream)), "orMallocAsync");
}

orError_t orFreeAsync(void* devPtr, orStream_t stream) {
  if (!devPtr) return orSuccess;
  return from_cuda(cudaFreeAsync(devPtr, as_cuda(stream)), "orFreeAsync");
}

orError_t orMemPoolTrim(size_t keep_bytes) {
  int dev = 0;
  MCPU_CUDA_TRY(cudaGetDevice(&dev), "orMemPoolTrim");
  cudaMemPool_t pool;
  MCPU_CUDA_TRY(cudaDeviceGetDefaultMemPool(&pool, dev), "orMemPoolTrim");
  MCPU_CUDA_TRY(cudaDeviceSynchronize(), "orMemPoolTrim");
  return from_cuda(cudaMemPoolTrimTo(pool, keep_bytes), "orMemPoolTrim");
}

orError_t mcpu_mem_get_info(int device, size_t* free_bytes, size_t* total_bytes) {
  MCPU_ARG_CHECK(free_bytes && total_bytes, "mem_get_info: NULL output");
  int prev = 0;
  MCPU_CUDA_TRY(cudaGetDevice(&prev), "mem_get_info");
  if (device >= 0 && device != prev) MCPU_CUDA_TRY(cudaSetDevice(device), "mem_get_info");
  const cudaError_t e = cudaMemGetInfo(free_bytes, total_bytes);
  if (device >= 0 && device != prev) cudaSetDevice(prev);
  return from_cuda(e, "mem_get_info");
}

orError_t mcpu_mem_pool_reserved(int device, uint64_t* current, uint64_t* peak) {
  MCPU_ARG_CHECK(current && peak, "mem_pool_reserved: NULL output");
  int dev = device;
  if (dev < 0) MCPU_CUDA_TRY(cudaGetDevice(&dev), "mem_pool_reserved");
  cudaMemPool_t pool;
  MCPU_CUDA_TRY(cudaDeviceGetDefaultMemPool(&pool, dev), "mem_pool_reserved");
  unsigned long long c = 0, h = 0;  // the attributes are 64-bit
  MCPU_CUDA_TRY(cudaMemPoolGetAttribute(pool, cudaMemPoolAttrReservedMemCurrent, &c), "mem_pool_reserved");
  MCPU_CUDA_TRY(cudaMemPoolGetAttribute(pool, cudaMemPoolAttrReservedMemHigh, &h), "mem_pool_reserved");
  *current = c;
  *peak = h;
  return orSuccess;
}

orError_t mcpu_copy_strided(const void* src, int src_dtype, void* dst, int dst_dtype, int ndim,
                            const int64_t* sizes, const int64_t* src_strides,
                            const int64_t* dst_strides, orStream_t stream) {
  MCPU_ARG_CHECK(tensor::valid_dtype(src_dtype) && tensor::valid_dtype(dst_dtype),
                 "copy: unsupported dtype (%d -> %d)", src_dtype, dst_dtype);
  MCPU_ARG_CHECK(ndim >= 0 && ndim <= tensor::kMaxDims, "copy: at most %d dimensions", tensor::kMaxDims);
  tensor::Strided s;
  s.ndim = ndim;
  long long n = 1;
  for (int d = 0; d < ndim; ++d) {
    MCPU_ARG_CHECK(sizes[d] >= 0, "copy: negative size");
    s.sizes[d] = sizes[d];
    s.src[d] = src_strides[d];
    s.dst[d] = dst_strides[d];
    n *= sizes[d];
  }
  if (n == 0) return orSuccess;
  MCPU_ARG_CHECK(src && dst, "copy: NULL tensor pointer");
  return from_cuda(tensor::launch_copy(src_dtype, dst_dtype, src, dst, s, n, tensor::grid_for(n), as_cuda(stream)),
                   "copy launch");
}

orError_t mcpu_fill(void* dst, int dtype, int ndim, const int64_t* sizes, const int64_t* strides,
                    double fvalue, int64_t ivalue, int value_is_float, orStream_t stream) {
  MCPU_ARG_CHECK(tensor::valid_dtype(dtype), "fill: unsupported dtype %d", dtype);
  MCPU_ARG_CHECK(ndim >= 0 && ndim <= tensor::kMaxDims, "fill: at most %d dimensions", tensor::kMaxDims);
  tensor::Strided s;
  s.ndim = ndim;
  long long n = 1;
  for (int d = 0; d < ndim; ++d) {
    s.sizes[d] = sizes[d];
    s.src[d] = 0;
    s.dst[d] = strides[d];
    n *= sizes[d];
  }
  if (n == 0) return orSuccess;
  MCPU_ARG_CHECK(dst != nullptr, "fill: NULL tensor pointer");
  tensor::Val v;
  v.is_fp = value_is_float != 0;
  v.d = fvalue;
  v.i = ivalue;
  cudaStream_t st = as_cuda(stream);
  const int blocks = tensor::grid_for(n);
  switch (dtype) {
#define CASE(D, ...)                                                  \
  case D:                                                             \
    tensor::fill_kernel<D><<<blocks, 256, 0, st>>>(dst, s, n, v);    \
    break;
    MCPU_DTYPE_CASES(CASE)
#undef CASE
  }
  return from_cuda(cudaGetLastError(), "fill launch");
}

orError_t mcpu_sigmoid(void* out, const void* x, int64_t n, int dtype, orStream_t stream) {
  MCPU_ARG_CHECK(dtype == MCPU_FLOAT32 || dtype == MCPU_BFLOAT16, "sigmoid: float32 or bfloat16 only");
  if (n == 0) return orSuccess;
  MCPU_ARG_CHECK(out && x, "sigmoid: NULL tensor pointer");
  const int blocks = tensor::grid_for(n);
  if (dtype == MCPU_FLOAT32) tensor::sigmoid_kernel<MCPU_FLOAT32><<<blocks, 256, 0, as_cuda(stream)>>>(x, out, n);
  else tensor::sigmoid_kernel<MCPU_BFLOAT16><<<blocks, 256, 0, as_cuda(stream)>>>(x, out, n);
  return from_cuda(cudaGetLastError(), "sigmoid launch");
}

orError_t mcpu_silu(void* out, const void* x, int64_t n, int dtype, orStream_t stream) {
  MCPU_ARG_CHECK(dtype == MCPU_FLOAT32 || dtype == MCPU_BFLOAT16, "silu: float32 or bfloat16 only");
  if (n == 0) return orSuccess;
  MCPU_ARG_CHECK(out && x, "silu: NULL tensor pointer");
  const int blocks = tensor::grid_for(n);
  if (dtype == MCPU_FLOAT32) tensor::silu_kernel<MCPU_FLOAT32><<<blocks, 256, 0, as_cuda(stream)>>>(x, out, n);
  else tensor::silu_kernel<MCPU_BFLOAT16><<<blocks, 256, 0, as_cuda(stream)>>>(x, out, n);
  return from_cuda(cudaGetLastError(), "silu launch");
}

orError_t mcpu_mul(void* out, const void* a, const void* b, int64_t n, int dtype, orStream_t stream) {
  MCPU_ARG_CHECK(dtype == MCPU_FLOAT32 || dtype == MCPU_BFLOAT16, "mul: float32 or bfloat16 only");
  if (n == 0) return orSuccess;
  MCPU_ARG_CHECK(out && a && b, "mul: NULL tensor pointer");
  const int blocks = tensor::grid_for(n);
  if (dtype == MCPU_FLOAT32) tensor::mul_kernel<MCPU_FLOAT32><<<blocks, 256, 0, as_cuda(stream)>>>(a, b, out, n);
  else tensor::mul_kernel<MCPU_BFLOAT16><<<blocks, 256, 0, as_cuda(stream)>>>(a, b, out, n);
  return from_cuda(cudaGetLastError(), "mul launch");
}

}  // extern "C"
