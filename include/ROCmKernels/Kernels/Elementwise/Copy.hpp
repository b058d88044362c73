// Streaming device copy used by the benchmark harness for its memory ceilings. Same interface
// as ROCmKernels.Kernels/include/ROCmKernels/Kernels/Elementwise/Copy.hpp (Copy(source, destination, count, stream)).
#pragma once

#include <cstddef>
#include <hip/hip_runtime.h>

namespace ROCmKernels::Kernels {
    /// destination[i] = source[i] for i < count; throws HipError on a launch error.
    void Copy(const float *source, float *destination, std::size_t count, hipStream_t stream = nullptr);
} // namespace ROCmKernels::Kernels
