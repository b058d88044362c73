// Error type and check macro shared by the C++ wrappers, the tests and the benchmark harness.
// Same interface as ROCmKernels.Common/include/ROCmKernels/Common/Error.hpp:14-45 (HipError with
// Status(), ThrowHipError, ROCMKERNELS_HIP_CHECK); hipError_t is cudaError_t through the shim.
#pragma once

#include <hip/hip_runtime.h>

#include <stdexcept>
#include <string>

namespace ROCmKernels {
    /// Thrown when a runtime call or a library entry point returns a non-zero status.
    class HipError final : public std::runtime_error {
        hipError_t m_status;

      public:
        HipError(hipError_t status, const std::string &message) : std::runtime_error(message), m_status(status) {}

        [[nodiscard]] hipError_t Status() const noexcept { return this->m_status; }
    };

    /// Formats "<expression> -> <error text> (file:line)" and throws it as a HipError.
    [[noreturn]] inline void ThrowHipError(hipError_t status, const char *expression, const char *file, const int line) {
        std::string text = std::string("runtime call failed: ") + expression + " -> " + hipGetErrorString(status) +
                " (" + file + ":" + std::to_string(line) + ")";
        throw HipError(status, text);
    }
} // namespace ROCmKernels

#define ROCMKERNELS_HIP_CHECK(expression)                                                                   \
    do {                                                                                                    \
        const hipError_t rocmkernelsCheckedStatus = static_cast<hipError_t>(expression);                    \
        if (rocmkernelsCheckedStatus != hipSuccess)                                                         \
            ::ROCmKernels::ThrowHipError(rocmkernelsCheckedStatus, #expression, __FILE__, __LINE__);        \
    } while (false)
