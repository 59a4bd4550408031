/*
 * Device runtime C-ABI of the mcpu device, backed by the CUDA runtime on
 * B200 (sm_100a).
 *
 * Drop-in for third_party/openreg/include/openreg.h of kzwrime/torch_mcpu:
 * the same function names, argument meaning, enum values and ownership rules
 * (the caller owns every stream, event and allocation).  What changes is the
 * backing store: "device" memory is HBM (cudaMalloc), streams are CUDA
 * streams and events are CUDA events.
 *
 * Replaced entry points (reference file:line):
 *   orError_t enum ................ openreg.h:15-20 (values 0-3 kept; 4 added)
 *   orMalloc..orMemoryProtect ..... openreg.h:56-71
 *   orGetDeviceCount..orDeviceSynchronize  openreg.h:74-79
 *   orStreamCreate*..orStreamWaitEvent     openreg.h:82-92
 *   orEvent*  ..................... openreg.h:95-103
 *
 * Behaviour notes:
 *  - orStream_t is a cudaStream_t (a NULL stream is CUDA's legacy default
 *    stream), so a caller may pass torch.cuda.current_stream().cuda_stream.
 *  - orStreamSynchronize / orEventSynchronize honour
 *    TORCH_MCPU_STREAM_SYNC_TIMEOUT_MS like the reference
 *    (third_party/openreg/csrc/stream.cpp:229-240, 321-349): they poll and
 *    return orErrorTimeout after the deadline instead of blocking forever.
 *  - orMemoryProtect / orMemoryUnprotect return orSuccess and do nothing:
 *    HBM is not host-addressable, so there is no page protection to toggle.
 *  - orDeviceGetStreamPriorityRange keeps the reference's convention
 *    (least = 1, greatest = 0); priority 0 maps to CUDA's greatest priority.
 */
#pragma once

#include <stddef.h>

#ifdef _WIN32
#define OPENREG_EXPORT __declspec(dllexport)
#else
#define OPENREG_EXPORT __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum orError_t {
  orSuccess = 0,
  orErrorUnknown = 1,
  orErrorNotReady = 2,
  orErrorTimeout = 3,
  /* Not in the reference: argument validation failures of the op entry
   * points (the reference raises c10::Error for these). */
  orErrorInvalidValue = 4
} orError_t;

typedef enum orMemcpyKind {
  orMemcpyHostToHost = 0,
  orMemcpyHostToDevice = 1,
  orMemcpyDeviceToHost = 2,
  orMemcpyDeviceToDevice = 3
} orMemcpyKind;

typedef enum orMemoryType {
  orMemoryTypeUnmanaged = 0,
  orMemoryTypeHost = 1,
  orMemoryTypeDevice = 2
} orMemoryType;

struct orPointerAttributes {
  orMemoryType type;
  int device;
  void* pointer;
};

typedef enum orEventFlags {
  orEventDisableTiming = 0x0,
  orEventEnableTiming = 0x1,
} orEventFlags;

struct orStream;
struct orEvent;
typedef struct orStream* orStream_t;
typedef struct orEvent* orEvent_t;

typedef enum orStreamCreateFlags {
  orStreamDefault = 0x1,
} orStreamCreateFlags;

/* Memory */
OPENREG_EXPORT orError_t orMalloc(void** devPtr, size_t size);
OPENREG_EXPORT orError_t orFree(void* devPtr);
OPENREG_EXPORT orError_t orMallocHost(void** hostPtr, size_t size);
OPENREG_EXPORT orError_t orFreeHost(void* hostPtr);
OPENREG_EXPORT orError_t orMemcpy(void* dst, const void* src, size_t count,
                                  orMemcpyKind kind);
OPENREG_EXPORT orError_t orMemcpyAsync(void* dst, const void* src,
                                       size_t count, orMemcpyKind kind,
                                       orStream_t stream);
OPENREG_EXPORT orError_t orPointerGetAttributes(
    struct orPointerAttributes* attributes, const void* ptr);
OPENREG_EXPORT orError_t orMemoryUnprotect(void* devPtr);
OPENREG_EXPORT orError_t orMemoryProtect(void* devPtr);

/* Stream-ordered allocation (not in the reference's C-ABI; it backs the
 * caching allocator of csrc/runtime/DeviceCachingAllocator.cpp):
 * cudaMallocAsync / cudaFreeAsync on the device's default memory pool, whose
 * release threshold is raised so freed memory stays cached; orMemPoolTrim
 * returns cached memory above keep_bytes to the driver (empty_cache). */
OPENREG_EXPORT orError_t orMallocAsync(void** devPtr, size_t size, orStream_t stream);
OPENREG_EXPORT orError_t orFreeAsync(void* devPtr, orStream_t stream);
OPENREG_EXPORT orError_t orMemPoolTrim(size_t keep_bytes);

/* Device */
OPENREG_EXPORT orError_t orGetDeviceCount(int* count);
OPENREG_EXPORT orError_t orSetDevice(int device);
OPENREG_EXPORT orError_t orGetDevice(int* device);
OPENREG_EXPORT orError_t orDeviceGetStreamPriorityRange(int* leastPriority,
                                                        int* greatestPriority);
OPENREG_EXPORT orError_t orDeviceSynchronize(void);

/* Stream */
OPENREG_EXPORT orError_t orStreamCreateWithPriority(orStream_t* stream,
                                                    unsigned int flags,
                                                    int priority);
OPENREG_EXPORT orError_t orStreamCreate(orStream_t* stream);
OPENREG_EXPORT orError_t orStreamGetPriority(orStream_t stream, int* priority);
OPENREG_EXPORT orError_t orStreamDestroy(orStream_t stream);
OPENREG_EXPORT orError_t orStreamQuery(orStream_t stream);
OPENREG_EXPORT orError_t orStreamSynchronize(orStream_t stream);
OPENREG_EXPORT orError_t orStreamWaitEvent(orStream_t stream, orEvent_t event,
                                           unsigned int flags);

/* Event */
OPENREG_EXPORT orError_t orEventCreateWithFlags(orEvent_t* event,
                                                unsigned int flags);
OPENREG_EXPORT orError_t orEventCreate(orEvent_t* event);
OPENREG_EXPORT orError_t orEventDestroy(orEvent_t event);
OPENREG_EXPORT orError_t orEventRecord(orEvent_t event, orStream_t stream);
OPENREG_EXPORT orError_t orEventSynchronize(orEvent_t event);
OPENREG_EXPORT orError_t orEventQuery(orEvent_t event);
OPENREG_EXPORT orError_t orEventElapsedTime(float* ms, orEvent_t start,
                                            orEvent_t end);

#ifdef __cplusplus
}  // extern "C"
#endif
