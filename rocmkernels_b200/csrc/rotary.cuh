// Rotary embedding of 32-wide heads (ROCmKernels.Kernels/src/Positional/Rotary.hip:10-42): feature
// c of a head rotates with feature c + 16 by the per-(batch, token) tables cos and sin.
#pragma once

#include <cuda_runtime.h>

namespace rk {

// One (low, high) pair, with explicit roundings so that the standalone kernel and the attention
// prologue produce the same bits:
//   forward  lo' = lo cos_lo - hi sin_lo,  hi' = hi cos_hi + lo sin_hi   (Rotary.hip:37-40)
//   backward lo' = lo cos_lo + hi sin_hi,  hi' = hi cos_hi - lo sin_lo   (Rotary.hip:32-35, the
//            transposed rotation, i.e. the gradient of the forward)
// each as one product rounded to FP32 and one fused multiply-add.
template <bool kBackward>
__device__ __forceinline__ void rotate_pair(float lo, float hi, float cos_lo, float cos_hi, float sin_lo, float sin_hi,
                                            float &out_lo, float &out_hi) {
    if (kBackward) {
        out_lo = __fmaf_rn(lo, cos_lo, __fmul_rn(hi, sin_hi));
        out_hi = __fmaf_rn(hi, cos_hi, -__fmul_rn(lo, sin_lo));
    } else {
        out_lo = __fmaf_rn(lo, cos_lo, -__fmul_rn(hi, sin_lo));
        out_hi = __fmaf_rn(hi, cos_hi, __fmul_rn(lo, sin_hi));
    }
}

}  // namespace rk
