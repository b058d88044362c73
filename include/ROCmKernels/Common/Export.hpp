// Visibility of the library's C entry points (interface of ROCmKernels.Common/include/ROCmKernels/Common/Export.hpp:5-11).
#pragma once

#if defined(_WIN32)
#define ROCMKERNELS_EXPORT __declspec(dllexport)
#else
#define ROCMKERNELS_EXPORT __attribute__((visibility("default")))
#endif
