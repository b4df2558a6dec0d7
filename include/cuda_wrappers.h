/*
 * cuda_wrappers.h -- CUDA runtime shim (libcudawrap.so), drop-in for the
 * reference engine's csrc/cuda_wrappers.h.
 *
 * The enum values, typedefs and the 22 entry points below are the binary
 * interface the Terra engine links against (src/terra/engine.t:27-30 loads
 * the library, :32-100 re-declares the symbols), so they are kept exactly as
 * the reference declares them (csrc/cuda_wrappers.h:11-45).  The
 * implementation (time_b200/csrc/cuda_wrappers.cu) is new.
 *
 * cwStream_t carries a cudaStream_t; every other library in this build takes
 * streams in this form (csrc/cuda_wrappers.h:20).
 */
#ifndef CUDA_WRAPPERS_H
#define CUDA_WRAPPERS_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* csrc/cuda_wrappers.h:11-18 */
typedef enum {
    CW_SUCCESS = 0,
    CW_ERROR_INVALID_VALUE = 1,
    CW_ERROR_OUT_OF_MEMORY = 2,
    CW_ERROR_NOT_INITIALIZED = 3,
    CW_ERROR_DEINITIALIZED = 4,
    CW_ERROR_UNKNOWN = 999
} cwError_t;

/* csrc/cuda_wrappers.h:20-22 */
typedef void* cwStream_t;
typedef void* cwEvent_t;
typedef uint64_t cwDevicePtr_t;

/* csrc/cuda_wrappers.h:24 */ cwError_t cwInit(void);
/* csrc/cuda_wrappers.h:25 */ cwError_t cwSetDevice(int device);
/* csrc/cuda_wrappers.h:26 */ cwError_t cwGetDevice(int* device);
/* csrc/cuda_wrappers.h:27 */ cwError_t cwGetDeviceCount(int* count);
/* csrc/cuda_wrappers.h:28 */ cwError_t cwDeviceSynchronize(void);
/* csrc/cuda_wrappers.h:29 */ cwError_t cwMalloc(cwDevicePtr_t* ptr, size_t size);
/* csrc/cuda_wrappers.h:30 */ cwError_t cwFree(cwDevicePtr_t ptr);
/* csrc/cuda_wrappers.h:31 */ cwError_t cwMemcpyH2D(cwDevicePtr_t dst, const void* src, size_t size);
/* csrc/cuda_wrappers.h:32 */ cwError_t cwMemcpyD2H(void* dst, cwDevicePtr_t src, size_t size);
/* csrc/cuda_wrappers.h:33 */ cwError_t cwMemcpyD2D(cwDevicePtr_t dst, cwDevicePtr_t src, size_t size);
/* csrc/cuda_wrappers.h:34 */ cwError_t cwMemset(cwDevicePtr_t ptr, int value, size_t size);
/* csrc/cuda_wrappers.h:35 */ cwError_t cwStreamCreate(cwStream_t* stream);
/* csrc/cuda_wrappers.h:36 */ cwError_t cwStreamDestroy(cwStream_t stream);
/* csrc/cuda_wrappers.h:37 */ cwError_t cwStreamSynchronize(cwStream_t stream);
/* csrc/cuda_wrappers.h:38 */ cwError_t cwEventCreate(cwEvent_t* event);
/* csrc/cuda_wrappers.h:39 */ cwError_t cwEventDestroy(cwEvent_t event);
/* csrc/cuda_wrappers.h:40 */ cwError_t cwEventRecord(cwEvent_t event, cwStream_t stream);
/* csrc/cuda_wrappers.h:41 */ cwError_t cwEventSynchronize(cwEvent_t event);
/* csrc/cuda_wrappers.h:42 */ cwError_t cwEventElapsedTime(float* ms, cwEvent_t start, cwEvent_t end);
/* csrc/cuda_wrappers.h:43 */ size_t cwGetFreeMemory(void);
/* csrc/cuda_wrappers.h:44 */ size_t cwGetTotalMemory(void);
/* csrc/cuda_wrappers.h:45 */ const char* cwGetErrorString(cwError_t error);

#ifdef __cplusplus
}
#endif

#endif /* CUDA_WRAPPERS_H */
