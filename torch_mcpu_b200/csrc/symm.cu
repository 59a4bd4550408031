// Symmetric windows: a device buffer per rank that every rank of the box
// maps through CUDA IPC, so kernels store into and load from the other GPUs'
// buffers over NVLink (mcpu_mm_allreduce).  The host side (torch_mcpu_b200/
// symm.py) exchanges the handles through the process group's store.
#include <string.h>

#include "common.cuh"

using namespace mcpu;

static_assert(sizeof(cudaIpcMemHandle_t) == MCPU_SYMM_HANDLE_BYTES, "IPC handle size");

extern "C" orError_t mcpu_symm_alloc(uint64_t bytes, void** ptr, uint8_t* handle) {
  MCPU_ARG_CHECK(ptr != nullptr && handle != nullptr, "symm_alloc: NULL output");
  MCPU_ARG_CHECK(bytes > 0, "symm_alloc: empty window");
  void* p = nullptr;
  MCPU_CUDA_TRY(cudaMalloc(&p, bytes), "symm_alloc cudaMalloc");
  cudaError_t st = cudaMemset(p, 0, bytes);
  if (st == cudaSuccess) st = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (st == cudaSuccess) st = cudaIpcGetMemHandle(&h, p);
  if (st != cudaSuccess) {
    cudaFree(p);
    return from_cuda(st, "symm_alloc");
  }
  memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return orSuccess;
}

extern "C" orError_t mcpu_symm_open(const uint8_t* handle, void** ptr) {
  MCPU_ARG_CHECK(ptr != nullptr && handle != nullptr, "symm_open: NULL argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  MCPU_CUDA_TRY(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess), "symm_open");
  return orSuccess;
}

extern "C" orError_t mcpu_symm_close(void* ptr) {
  MCPU_ARG_CHECK(ptr != nullptr, "symm_close: NULL pointer");
  return from_cuda(cudaIpcCloseMemHandle(ptr), "symm_close");
}

extern "C" orError_t mcpu_symm_free(void* ptr) {
  MCPU_ARG_CHECK(ptr != nullptr, "symm_free: NULL pointer");
  return from_cuda(cudaFree(ptr), "symm_free");
}

extern "C" orError_t mcpu_symm_clear(void* ptr, uint64_t bytes, orStream_t stream) {
  MCPU_ARG_CHECK(ptr != nullptr, "symm_clear: NULL pointer");
  return from_cuda(cudaMemsetAsync(ptr, 0, bytes, as_cuda(stream)), "symm_clear");
}
