// Element strides of a [batch][head][token] tensor. Replaces
// ROCmKernels.Kernels/include/ROCmKernels/Kernels/Strides.hpp:5-9; the type is the C ABI struct
// RocmKernelsStrides so the extern "C" declarations and the C++ wrappers share one definition.
#pragma once

#include <rocmkernels_attention.h>

namespace ROCmKernels::Kernels {
    using Strides = ::RocmKernelsStrides;
} // namespace ROCmKernels::Kernels
