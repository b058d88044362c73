// C++ interface of the generic forward; same name, signature and default stream as
// ROCmKernels.Kernels/include/ROCmKernels/Kernels/Generic/AttentionGeneric.hpp:15-25. The extern "C"
// entry point is declared once, in rocmkernels_attention.h, with the DType passed as its byte.
#pragma once

#include <ROCmKernels/Common/Error.hpp>
#include <ROCmKernels/Common/Export.hpp>
#include <ROCmKernels/Kernels/DType.hpp>
#include <ROCmKernels/Kernels/Strides.hpp>

#include <hip/hip_runtime.h>
#include <rocmkernels_attention.h>

namespace ROCmKernels::Kernels {
    /// Windowed flash attention forward for 16-, 32- or 64-wide heads.
    ///
    /// mask is [batch][keys]. radius < 0 attends globally. lse receives {row maximum, exponent sum} per (batch, head, query).
    /// q, k and v use qs, ks and vs; output uses os. Throws HipError on a non-zero status.
    inline void AttentionGenericForward(const void *q, const void *k, const void *v, const bool *mask, void *output, float *lse,
            const int batch, const int heads, const int queries, const int keys, const int headWidth, const int radius, const Strides &qs,
            const Strides &ks, const Strides &vs, const Strides &os, const DType dtype, hipStream_t stream = nullptr) {
        ROCMKERNELS_HIP_CHECK(attention_generic_forward(q, k, v, mask, output, lse, batch, heads, queries, keys, headWidth, radius, qs, ks,
                vs, os, static_cast<RocmKernelsDType>(dtype), stream));
    }
} // namespace ROCmKernels::Kernels
