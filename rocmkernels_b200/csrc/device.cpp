// Device queries (interface of ROCmKernels.Common/src/Device.cpp:10-43) over the CUDA runtime.
#include <ROCmKernels/Common/Device.hpp>
#include <ROCmKernels/Common/Error.hpp>

#include "context.h"

// The harness links these C++ symbols from the shared library.
#pragma GCC visibility push(default)
namespace ROCmKernels {

int GetDeviceCount() {
    int count = 0;
    ROCMKERNELS_HIP_CHECK(hipGetDeviceCount(&count));
    return count;
}

DeviceInfo QueryDevice(const int deviceIndex) {
    hipDeviceProp_t properties{};
    ROCMKERNELS_HIP_CHECK(hipGetDeviceProperties(&properties, deviceIndex));
    DeviceInfo info{};
    info.name = properties.name;
    info.gcnArchName = properties.gcnArchName;
    info.totalGlobalMemory = static_cast<std::uint64_t>(properties.totalGlobalMem);
    info.computeUnitCount = static_cast<std::uint32_t>(properties.multiProcessorCount);
    int clockKHz = 0;
    ROCMKERNELS_HIP_CHECK(cudaDeviceGetAttribute(&clockKHz, cudaDevAttrClockRate, deviceIndex));
    info.clockRateKHz = static_cast<std::uint32_t>(clockKHz);
    info.warpSize = static_cast<std::uint32_t>(properties.warpSize);
    ROCMKERNELS_HIP_CHECK(hipRuntimeGetVersion(&info.runtimeVersion));
    ROCMKERNELS_HIP_CHECK(hipDriverGetVersion(&info.driverVersion));
    return info;
}

void SynchronizeDevice(const int deviceIndex) {
    ROCMKERNELS_HIP_CHECK(hipSetDevice(deviceIndex));
    ROCMKERNELS_HIP_CHECK(hipDeviceSynchronize());
}

void ResetDevice(const int deviceIndex) {
    ROCMKERNELS_HIP_CHECK(hipSetDevice(deviceIndex));
    // Per-context caches (kernel attributes, the static delta array's address) are dropped even
    // if the driver were to hand the next context the same id.
    rk::invalidate_context_caches();
    ROCMKERNELS_HIP_CHECK(hipDeviceReset());
}

}  // namespace ROCmKernels
#pragma GCC visibility pop
