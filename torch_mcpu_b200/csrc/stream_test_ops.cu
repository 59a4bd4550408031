// Device side of the reference's stream test ops (csrc/aten/native/Extra.cpp:
// 255-296 of kzwrime/torch_mcpu: stream_sleep_fill_, stream_sleep_copy_,
// first_element_int).  There, the "kernel" is a host lambda on a worker
// thread that sleeps, then fills or copies host memory; here it is a device
// kernel that waits on the GPU's global timer, then fills or copies, so
// that stream ordering, stream waits and synchronisation are observable the
// same way.  The wait is bounded twice: by the requested time and by an
// iteration limit.
#include <mutex>

#include "common.cuh"

namespace mcpu {
namespace {

constexpr int kSleepThreads = 256;
constexpr long long kMaxSleepMs = 60000;

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// One CTA: thread 0 waits sleep_ms on the global timer (in steps of at most
// 100 us, at most 10000 steps per ms), then every thread fills or copies.
__global__ void __launch_bounds__(kSleepThreads) sleep_then_kernel(int64_t* dst, const int64_t* src,
                                                                   long long n, int64_t value,
                                                                   long long sleep_ms) {
  if (threadIdx.x == 0 && sleep_ms > 0) {
    const unsigned long long end = global_ns() + static_cast<unsigned long long>(sleep_ms) * 1000000ull;
    const unsigned long long limit = static_cast<unsigned long long>(sleep_ms) * 10000ull;
    for (unsigned long long i = 0; i < limit && global_ns() < end; ++i) __nanosleep(100000);
  }
  __syncthreads();
  for (long long i = threadIdx.x; i < n; i += kSleepThreads) dst[i] = src ? src[i] : value;
}

constexpr int kMaxDevices = 64;
std::mutex g_read_mutex;
cudaStream_t g_read_stream[kMaxDevices] = {};

}  // namespace
}  // namespace mcpu

using namespace mcpu;

extern "C" orError_t mcpu_stream_sleep_fill_i64(int64_t* x, int64_t numel, int64_t value, int64_t sleep_ms,
                                                orStream_t stream) {
  MCPU_ARG_CHECK(x != nullptr && numel > 0, "stream_sleep_fill_: empty or NULL tensor");
  MCPU_ARG_CHECK(sleep_ms >= 0 && sleep_ms <= kMaxSleepMs, "stream_sleep_fill_: sleep_ms %lld outside 0..%lld",
                 static_cast<long long>(sleep_ms), kMaxSleepMs);
  sleep_then_kernel<<<1, kSleepThreads, 0, as_cuda(stream)>>>(x, nullptr, numel, value, sleep_ms);
  return from_cuda(cudaGetLastError(), "stream_sleep_fill_ launch");
}

extern "C" orError_t mcpu_stream_sleep_copy_i64(int64_t* dst, const int64_t* src, int64_t numel, int64_t sleep_ms,
                                                orStream_t stream) {
  MCPU_ARG_CHECK(dst != nullptr && src != nullptr && numel > 0, "stream_sleep_copy_: empty or NULL tensor");
  MCPU_ARG_CHECK(sleep_ms >= 0 && sleep_ms <= kMaxSleepMs, "stream_sleep_copy_: sleep_ms %lld outside 0..%lld",
                 static_cast<long long>(sleep_ms), kMaxSleepMs);
  sleep_then_kernel<<<1, kSleepThreads, 0, as_cuda(stream)>>>(dst, src, numel, 0, sleep_ms);
  return from_cuda(cudaGetLastError(), "stream_sleep_copy_ launch");
}

extern "C" orError_t mcpu_read_i64_now(const int64_t* src, int64_t* out) {
  MCPU_ARG_CHECK(src != nullptr && out != nullptr, "first_element_int: NULL pointer");
  int dev = 0;
  MCPU_CUDA_TRY(cudaGetDevice(&dev), "first_element_int");
  MCPU_ARG_CHECK(dev >= 0 && dev < kMaxDevices, "first_element_int: device %d out of range", dev);
  cudaStream_t s;
  {
    std::lock_guard<std::mutex> lock(g_read_mutex);
    if (g_read_stream[dev] == nullptr)
      MCPU_CUDA_TRY(cudaStreamCreateWithFlags(&g_read_stream[dev], cudaStreamNonBlocking), "first_element_int");
    s = g_read_stream[dev];
  }
  MCPU_CUDA_TRY(cudaMemcpyAsync(out, src, sizeof(int64_t), cudaMemcpyDeviceToHost, s), "first_element_int");
  return from_cuda(cudaStreamSynchronize(s), "first_element_int");
}
