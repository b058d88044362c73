// HIP half-precision header mapped onto CUDA's (__half and its intrinsics).
#pragma once
#include <cuda_fp16.h>
