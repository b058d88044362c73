// HIP-to-CUDA runtime shim.
//
// Maps the HIP runtime names used by the attention interface, its C++ wrappers, the reference's
// attention tests and its benchmark harness onto the CUDA runtime, so that those sources compile
// unchanged for sm_100a. hipError_t is cudaError_t (hipSuccess == cudaSuccess == 0,
// hipErrorInvalidValue == cudaErrorInvalidValue == 1), hipStream_t is cudaStream_t. Only the
// subset those sources use is provided; anything else is a compile error, not a silent stub.
#pragma once

#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>

typedef cudaError_t hipError_t;
typedef cudaStream_t hipStream_t;
typedef cudaEvent_t hipEvent_t;
typedef cudaMemcpyKind hipMemcpyKind;

#define hipSuccess cudaSuccess
#define hipErrorInvalidValue cudaErrorInvalidValue
#define hipErrorOutOfMemory cudaErrorMemoryAllocation
#define hipErrorNotReady cudaErrorNotReady
#define hipMemcpyHostToDevice cudaMemcpyHostToDevice
#define hipMemcpyDeviceToHost cudaMemcpyDeviceToHost
#define hipMemcpyDeviceToDevice cudaMemcpyDeviceToDevice
#define hipMemcpyHostToHost cudaMemcpyHostToHost
#define hipMemcpyDefault cudaMemcpyDefault

/// cudaDeviceProp plus HIP's gcnArchName, which holds the CUDA architecture ("sm_100a").
struct hipDeviceProp_t : cudaDeviceProp {
    char gcnArchName[256];
};

inline const char *hipGetErrorString(hipError_t error) { return cudaGetErrorString(error); }
inline const char *hipGetErrorName(hipError_t error) { return cudaGetErrorName(error); }
inline hipError_t hipGetLastError() { return cudaGetLastError(); }
inline hipError_t hipPeekAtLastError() { return cudaPeekAtLastError(); }

inline hipError_t hipMalloc(void **pointer, size_t bytes) { return cudaMalloc(pointer, bytes); }
template <typename T> inline hipError_t hipMalloc(T **pointer, size_t bytes) {
    return cudaMalloc(reinterpret_cast<void **>(pointer), bytes);
}
inline hipError_t hipFree(void *pointer) { return cudaFree(pointer); }
inline hipError_t hipHostMalloc(void **pointer, size_t bytes, unsigned int = 0) { return cudaMallocHost(pointer, bytes); }
inline hipError_t hipHostFree(void *pointer) { return cudaFreeHost(pointer); }
inline hipError_t hipMemcpy(void *destination, const void *source, size_t bytes, hipMemcpyKind kind) {
    return cudaMemcpy(destination, source, bytes, kind);
}
inline hipError_t hipMemcpyAsync(void *destination, const void *source, size_t bytes, hipMemcpyKind kind,
        hipStream_t stream = nullptr) {
    return cudaMemcpyAsync(destination, source, bytes, kind, stream);
}
inline hipError_t hipMemset(void *destination, int value, size_t bytes) { return cudaMemset(destination, value, bytes); }
inline hipError_t hipMemsetAsync(void *destination, int value, size_t bytes, hipStream_t stream = nullptr) {
    return cudaMemsetAsync(destination, value, bytes, stream);
}

inline hipError_t hipDeviceSynchronize() { return cudaDeviceSynchronize(); }
inline hipError_t hipDeviceReset() { return cudaDeviceReset(); }
inline hipError_t hipSetDevice(int device) { return cudaSetDevice(device); }
inline hipError_t hipGetDevice(int *device) { return cudaGetDevice(device); }
inline hipError_t hipGetDeviceCount(int *count) { return cudaGetDeviceCount(count); }
inline hipError_t hipRuntimeGetVersion(int *version) { return cudaRuntimeGetVersion(version); }
inline hipError_t hipDriverGetVersion(int *version) { return cudaDriverGetVersion(version); }
inline hipError_t hipGetDeviceProperties(hipDeviceProp_t *properties, int device) {
    const hipError_t status = cudaGetDeviceProperties(static_cast<cudaDeviceProp *>(properties), device);
    if (status != cudaSuccess) return status;
    // Arch-specific "a" suffix: the library is built for sm_100a only.
    std::snprintf(properties->gcnArchName, sizeof(properties->gcnArchName), "sm_%d%d%s", properties->major,
            properties->minor, properties->major >= 9 ? "a" : "");
    return cudaSuccess;
}

inline hipError_t hipStreamCreate(hipStream_t *stream) { return cudaStreamCreate(stream); }
inline hipError_t hipStreamDestroy(hipStream_t stream) { return cudaStreamDestroy(stream); }
inline hipError_t hipStreamSynchronize(hipStream_t stream) { return cudaStreamSynchronize(stream); }

inline hipError_t hipEventCreate(hipEvent_t *event) { return cudaEventCreate(event); }
inline hipError_t hipEventDestroy(hipEvent_t event) { return cudaEventDestroy(event); }
inline hipError_t hipEventRecord(hipEvent_t event, hipStream_t stream = nullptr) { return cudaEventRecord(event, stream); }
inline hipError_t hipEventSynchronize(hipEvent_t event) { return cudaEventSynchronize(event); }
inline hipError_t hipEventElapsedTime(float *milliseconds, hipEvent_t start, hipEvent_t stop) {
    return cudaEventElapsedTime(milliseconds, start, stop);
}

#if defined(__CUDACC__)
/// hipLaunchKernelGGL(kernel, grid, block, sharedBytes, stream, args...) as a CUDA launch.
#define hipLaunchKernelGGL(kernel, grid, block, sharedBytes, stream, ...) \
    kernel<<<(grid), (block), (sharedBytes), (stream)>>>(__VA_ARGS__)
#endif
