// C++ interface of the 32-wide FP32 attention: the extern "C" entry points (declared in
// rocmkernels_attention.h) plus namespaced wrappers that throw ROCmKernels::HipError on a
// non-zero status. Same names, signatures and defaults as
// ROCmKernels.Kernels/include/ROCmKernels/Kernels/Attention/Attention.hpp:9-108, so callers
// written against the reference compile unchanged.
//
// Layouts: mask is [batch][keys]; radius < 0 attends globally. output is written at
// os.batch/os.head/os.token; lse ({row max of scaled scores, exponent sum} per row), delta and
// the gradients are packed [batch][head][query|key][32].
#pragma once

#include <ROCmKernels/Common/Error.hpp>
#include <ROCmKernels/Common/Export.hpp>
#include <ROCmKernels/Kernels/Strides.hpp>

#include <hip/hip_runtime.h>
#include <rocmkernels_attention.h>

namespace ROCmKernels::Kernels {
    inline void AttentionForward(const float *q, const float *k, const float *v, const bool *mask, float *output, float *lse, const int batch,
            const int heads, const int queries, const int keys, const int radius, const Strides &qs, const Strides &ks, const Strides &vs,
            const Strides &os, hipStream_t stream = nullptr) {
        ROCMKERNELS_HIP_CHECK(attention_fp32_forward(q, k, v, mask, output, lse, batch, heads, queries, keys, radius, qs, ks, vs, os, stream));
    }

    inline void AttentionForwardTiled(const float *q, const float *k, const float *v, const bool *mask, float *output, float *lse,
            const int batch, const int heads, const int queries, const int keys, const int radius, const Strides &qs, const Strides &ks,
            const Strides &vs, const Strides &os, hipStream_t stream = nullptr) {
        ROCMKERNELS_HIP_CHECK(attention_fp32_forward_tiled(q, k, v, mask, output, lse, batch, heads, queries, keys, radius, qs, ks, vs, os, stream));
    }

    /// delta receives sum(upstream * output) per query row.
    inline void AttentionBackward(const float *q, const float *k, const float *v, const bool *mask, const float *output, const float *lse,
            const float *upstream, float *gradient_q, float *gradient_k, float *gradient_v, float *delta, const int batch, const int heads,
            const int queries, const int keys, const int radius, const Strides &qs, const Strides &ks, const Strides &vs, const Strides &os,
            const Strides &us, hipStream_t stream = nullptr) {
        ROCMKERNELS_HIP_CHECK(attention_fp32_backward(q, k, v, mask, output, lse, upstream, gradient_q, gradient_k, gradient_v, delta, batch,
                heads, queries, keys, radius, qs, ks, vs, os, us, stream));
    }

    inline void AttentionBackwardTiled(const float *q, const float *k, const float *v, const bool *mask, const float *output,
            const float *lse, const float *upstream, float *gradient_q, float *gradient_k, float *gradient_v, float *delta, const int batch,
            const int heads, const int queries, const int keys, const int radius, const Strides &qs, const Strides &ks, const Strides &vs,
            const Strides &os, const Strides &us, hipStream_t stream = nullptr) {
        ROCMKERNELS_HIP_CHECK(attention_fp32_backward_tiled(q, k, v, mask, output, lse, upstream, gradient_q, gradient_k, gradient_v, delta,
                batch, heads, queries, keys, radius, qs, ks, vs, os, us, stream));
    }

    /// Softmax statistics only; no value reads and no output write.
    inline void AttentionStatistics(const float *q, const float *k, const bool *mask, float *lse, const int batch, const int heads,
            const int queries, const int keys, const int radius, const Strides &qs, const Strides &ks, hipStream_t stream = nullptr) {
        ROCMKERNELS_HIP_CHECK(attention_fp32_statistics(q, k, mask, lse, batch, heads, queries, keys, radius, qs, ks, stream));
    }

    inline void AttentionForwardTuned(const float *q, const float *k, const float *v, const bool *mask, float *output, float *lse,
            const int batch, const int heads, const int queries, const int keys, const int radius, const int group, const Strides &qs,
            const Strides &ks, const Strides &vs, const Strides &os, hipStream_t stream = nullptr) {
        ROCMKERNELS_HIP_CHECK(
                attention_fp32_forward_tuned(q, k, v, mask, output, lse, batch, heads, queries, keys, radius, group, qs, ks, vs, os, stream));
    }

    /// Flash forward: tcgen05/TMEM kernel with split-FP16 operands (kind::f16, ~22-bit products) on sm_100a.
    inline void AttentionForwardFlash(const float *q, const float *k, const float *v, const bool *mask, float *output, float *lse,
            const int batch, const int heads, const int queries, const int keys, const int radius, const Strides &qs, const Strides &ks,
            const Strides &vs, const Strides &os, hipStream_t stream = nullptr) {
        ROCMKERNELS_HIP_CHECK(attention_fp32_forward_flash(q, k, v, mask, output, lse, batch, heads, queries, keys, radius, qs, ks, vs, os, stream));
    }

    /// Variant selector 0 through 18 (the reference's tuning sweep ids).
    inline void AttentionForwardFlashTuned(const float *q, const float *k, const float *v, const bool *mask, float *output, float *lse,
            const int batch, const int heads, const int queries, const int keys, const int radius, const int variant, const Strides &qs,
            const Strides &ks, const Strides &vs, const Strides &os, hipStream_t stream = nullptr) {
        ROCMKERNELS_HIP_CHECK(
                attention_fp32_forward_flash_tuned(q, k, v, mask, output, lse, batch, heads, queries, keys, radius, variant, qs, ks, vs, os, stream));
    }

    inline void AttentionBackwardTuned(const float *q, const float *k, const float *v, const bool *mask, const float *output,
            const float *lse, const float *upstream, float *gradient_q, float *gradient_k, float *gradient_v, float *delta, const int batch,
            const int heads, const int queries, const int keys, const int radius, const int group, const Strides &qs, const Strides &ks,
            const Strides &vs, const Strides &os, const Strides &us, hipStream_t stream = nullptr) {
        ROCMKERNELS_HIP_CHECK(attention_fp32_backward_tuned(q, k, v, mask, output, lse, upstream, gradient_q, gradient_k, gradient_v, delta,
                batch, heads, queries, keys, radius, group, qs, ks, vs, os, us, stream));
    }
} // namespace ROCmKernels::Kernels
