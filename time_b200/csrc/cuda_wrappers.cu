// cuda_wrappers.cu -- libcudawrap: the CUDA-runtime shim the reference engine
// links (csrc/cuda_wrappers.h:24-45).  Same status mapping as the reference
// (csrc/cuda_wrappers.cu:7-17: invalid value, out of memory, not-ready ->
// not initialised, everything else unknown).  Failures are also reported on
// stderr, as the engine relies on that for diagnostics.
#include <cuda_runtime.h>
#include <cstdio>

#include "cuda_wrappers.h"

namespace {

bool g_initialized = false;

cwError_t to_cw(cudaError_t e) {
    switch (e) {
        case cudaSuccess: return CW_SUCCESS;
        case cudaErrorInvalidValue: return CW_ERROR_INVALID_VALUE;
        case cudaErrorMemoryAllocation: return CW_ERROR_OUT_OF_MEMORY;
        case cudaErrorNotReady: return CW_ERROR_NOT_INITIALIZED;
        default: return CW_ERROR_UNKNOWN;
    }
}

cwError_t report(cudaError_t e, const char* what) {
    if (e != cudaSuccess) std::fprintf(stderr, "%s failed: %s\n", what, cudaGetErrorString(e));
    return to_cw(e);
}

}  // namespace

extern "C" {

cwError_t cwInit(void) {
    if (g_initialized) return CW_SUCCESS;
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) return report(e, "cudaGetDeviceCount");
    if (n == 0) {
        std::fprintf(stderr, "no CUDA device\n");
        return CW_ERROR_NOT_INITIALIZED;
    }
    g_initialized = true;
    return CW_SUCCESS;
}

cwError_t cwSetDevice(int device) { return report(cudaSetDevice(device), "cudaSetDevice"); }
cwError_t cwGetDevice(int* device) { return to_cw(cudaGetDevice(device)); }
cwError_t cwGetDeviceCount(int* count) { return to_cw(cudaGetDeviceCount(count)); }
cwError_t cwDeviceSynchronize(void) { return report(cudaDeviceSynchronize(), "cudaDeviceSynchronize"); }

cwError_t cwMalloc(cwDevicePtr_t* ptr, size_t size) {
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, size);
    *ptr = (e == cudaSuccess) ? reinterpret_cast<cwDevicePtr_t>(p) : 0;
    return report(e, "cudaMalloc");
}

cwError_t cwFree(cwDevicePtr_t ptr) {
    if (ptr == 0) return CW_SUCCESS;
    return report(cudaFree(reinterpret_cast<void*>(ptr)), "cudaFree");
}

cwError_t cwMemcpyH2D(cwDevicePtr_t dst, const void* src, size_t size) {
    return report(cudaMemcpy(reinterpret_cast<void*>(dst), src, size, cudaMemcpyHostToDevice), "cudaMemcpy H2D");
}

cwError_t cwMemcpyD2H(void* dst, cwDevicePtr_t src, size_t size) {
    return report(cudaMemcpy(dst, reinterpret_cast<const void*>(src), size, cudaMemcpyDeviceToHost), "cudaMemcpy D2H");
}

cwError_t cwMemcpyD2D(cwDevicePtr_t dst, cwDevicePtr_t src, size_t size) {
    return report(cudaMemcpy(reinterpret_cast<void*>(dst), reinterpret_cast<const void*>(src), size,
                             cudaMemcpyDeviceToDevice), "cudaMemcpy D2D");
}

cwError_t cwMemset(cwDevicePtr_t ptr, int value, size_t size) {
    return report(cudaMemset(reinterpret_cast<void*>(ptr), value, size), "cudaMemset");
}

cwError_t cwStreamCreate(cwStream_t* stream) {
    cudaStream_t s = nullptr;
    // a blocking stream, as the reference creates: the engine relies on the
    // legacy default stream (cwMemcpy*) ordering against it.
    cudaError_t e = cudaStreamCreate(&s);
    *stream = (e == cudaSuccess) ? static_cast<cwStream_t>(s) : nullptr;
    return report(e, "cudaStreamCreate");
}

cwError_t cwStreamDestroy(cwStream_t stream) {
    if (!stream) return CW_SUCCESS;
    return to_cw(cudaStreamDestroy(static_cast<cudaStream_t>(stream)));
}

cwError_t cwStreamSynchronize(cwStream_t stream) {
    return report(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "cudaStreamSynchronize");
}

cwError_t cwEventCreate(cwEvent_t* event) {
    cudaEvent_t ev = nullptr;
    cudaError_t e = cudaEventCreate(&ev);
    *event = (e == cudaSuccess) ? static_cast<cwEvent_t>(ev) : nullptr;
    return to_cw(e);
}

cwError_t cwEventDestroy(cwEvent_t event) {
    if (!event) return CW_SUCCESS;
    return to_cw(cudaEventDestroy(static_cast<cudaEvent_t>(event)));
}

cwError_t cwEventRecord(cwEvent_t event, cwStream_t stream) {
    return to_cw(cudaEventRecord(static_cast<cudaEvent_t>(event), static_cast<cudaStream_t>(stream)));
}

cwError_t cwEventSynchronize(cwEvent_t event) { return to_cw(cudaEventSynchronize(static_cast<cudaEvent_t>(event))); }

cwError_t cwEventElapsedTime(float* ms, cwEvent_t start, cwEvent_t end) {
    return to_cw(cudaEventElapsedTime(ms, static_cast<cudaEvent_t>(start), static_cast<cudaEvent_t>(end)));
}

size_t cwGetFreeMemory(void) {
    size_t f = 0, t = 0;
    cudaMemGetInfo(&f, &t);
    return f;
}

size_t cwGetTotalMemory(void) {
    size_t f = 0, t = 0;
    cudaMemGetInfo(&f, &t);
    return t;
}

const char* cwGetErrorString(cwError_t error) {
    switch (error) {
        case CW_SUCCESS: return "Success";
        case CW_ERROR_INVALID_VALUE: return "Invalid value";
        case CW_ERROR_OUT_OF_MEMORY: return "Out of memory";
        case CW_ERROR_NOT_INITIALIZED: return "Not initialized";
        case CW_ERROR_DEINITIALIZED: return "Deinitialized";
        default: return "Unknown error";
    }
}

}  // extern "C"
