// Device queries. Same interface as ROCmKernels.Common/include/ROCmKernels/Common/Device.hpp:10-33;
// gcnArchName holds the CUDA architecture ("sm_100a") on this build.
#pragma once

#include <cstdint>
#include <string>

namespace ROCmKernels {
    struct DeviceInfo {
        std::string name;
        std::string gcnArchName;
        std::uint64_t totalGlobalMemory = 0;
        std::uint32_t computeUnitCount = 0;
        std::uint32_t clockRateKHz = 0;
        std::uint32_t warpSize = 0;
        int runtimeVersion = 0;
        int driverVersion = 0;
    };

    /// Number of visible devices; throws HipError when the runtime is unusable.
    [[nodiscard]] int GetDeviceCount();
    /// Properties of one device; throws HipError when it cannot be queried.
    [[nodiscard]] DeviceInfo QueryDevice(int deviceIndex = 0);
    /// Waits for all work queued on the device.
    void SynchronizeDevice(int deviceIndex = 0);
    /// Destroys this process's context on the device (cudaDeviceReset; other processes are unaffected).
    void ResetDevice(int deviceIndex = 0);
} // namespace ROCmKernels
