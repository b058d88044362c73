// Streaming float copy used by the benchmark harness for its memory ceilings. Same interface as
// ROCmKernels::Kernels::Copy (ROCmKernels.Kernels/src/Elementwise/Copy.hip); here a grid-stride
// kernel sized to the SM count, with 16-byte accesses when both pointers allow them.
#include <ROCmKernels/Common/Error.hpp>
#include <ROCmKernels/Kernels/Elementwise/Copy.hpp>

// The harness links these C++ symbols from the shared library.
#pragma GCC visibility push(default)

#include <cstdint>

namespace {

__global__ void copy_vector(const float4 *__restrict__ source, float4 *__restrict__ destination, std::size_t count) {
    const std::size_t stride = static_cast<std::size_t>(gridDim.x) * blockDim.x;
    for (std::size_t i = static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count; i += stride)
        destination[i] = __ldcs(source + i);
}

__global__ void copy_scalar(const float *__restrict__ source, float *__restrict__ destination, std::size_t count) {
    const std::size_t stride = static_cast<std::size_t>(gridDim.x) * blockDim.x;
    for (std::size_t i = static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count; i += stride)
        destination[i] = source[i];
}

unsigned grid_for(std::size_t work) {
    int device = 0, sms = 148;
    if (cudaGetDevice(&device) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    const std::size_t wanted = (work + 255) / 256;
    const std::size_t cap = static_cast<std::size_t>(sms) * 8;
    return static_cast<unsigned>(wanted < cap ? (wanted > 0 ? wanted : 1) : cap);
}

}  // namespace

namespace ROCmKernels::Kernels {
void Copy(const float *source, float *destination, std::size_t count, hipStream_t stream) {
    if (count == 0) return;
    const bool vector = count % 4 == 0 && (reinterpret_cast<std::uintptr_t>(source) & 15u) == 0 &&
                        (reinterpret_cast<std::uintptr_t>(destination) & 15u) == 0;
    if (vector) {
        copy_vector<<<grid_for(count / 4), 256, 0, stream>>>(reinterpret_cast<const float4 *>(source),
                                                             reinterpret_cast<float4 *>(destination), count / 4);
    } else {
        copy_scalar<<<grid_for(count), 256, 0, stream>>>(source, destination, count);
    }
    ROCMKERNELS_HIP_CHECK(cudaGetLastError());
}
}  // namespace ROCmKernels::Kernels
#pragma GCC visibility pop
