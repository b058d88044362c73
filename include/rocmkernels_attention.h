/*
 * C ABI of the B200 FP32 attention library (librocmkernels_attention.so).
 *
 * Every entry point below replaces the entry point of the same name in SecondNewtonLaw/ROCmKernels
 * (HIP, gfx1031) with an sm_100a CUDA implementation. Names, argument order, argument meaning,
 * validation and return codes are those of the reference, so existing callers (the reference's
 * Catch2 tests and benchmark cases through the C++ wrappers in ROCmKernels/Kernels/Attention/,
 * or a ctypes binding) work unchanged.
 *
 * Conventions shared by all entry points
 *   - q, k, v, upstream (dO) and output-in (O) are read at element
 *     b*strides.batch + h*strides.head + t*strides.token + c, feature stride 1.
 *   - output (O) is written with the `os` strides. lse ({row max of scaled scores, sum of
 *     exp(score - max)} per row), delta and the gradients are PACKED:
 *     lse [batch][heads][queries][2], delta [batch][heads][queries],
 *     gradient_q [batch][heads][queries][D], gradient_k/v [batch][heads][keys][D].
 *   - mask is [batch][keys] bytes; nonzero = key visible. Queries are never masked.
 *   - radius < 0 attends globally; otherwise query i sees key j only when |i - j| <= radius.
 *   - Scores are q.k / sqrt(D). A fully masked row gives O = 0 and lse = {-inf, 0}.
 *   - Returns 0 (cudaSuccess / hipSuccess) or an error code: 1 (cudaErrorInvalidValue, the same
 *     value as hipErrorInvalidValue) for null pointers, non-positive sizes, an invalid radius
 *     where the reference checks it, or an unknown selector; otherwise the launch error.
 *   - Calls are asynchronous and ordered on `stream` (NULL = the legacy default stream); the
 *     library never synchronizes, allocates nothing and keeps no state between calls, so it is
 *     reentrant across host threads and devices (the caller's current device is used).
 *   - All pointers are device pointers owned by the caller.
 *
 * Deliberate differences from the reference, all on inputs the reference does not handle:
 * entries whose HIP launcher validated nothing (tiled, tuned) validate like the simple entry
 * here instead of launching a kernel on null pointers.
 */
#ifndef ROCMKERNELS_ATTENTION_H
#define ROCMKERNELS_ATTENTION_H

#ifndef __cplusplus
#include <stdbool.h>
#endif

#if defined(_WIN32)
#define ROCMKERNELS_C_EXPORT __declspec(dllexport)
#else
#define ROCMKERNELS_C_EXPORT __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Element strides of a [batch][head][token] tensor; 3 ints passed by value.
 * Replaces ROCmKernels::Kernels::Strides (ROCmKernels.Kernels/include/ROCmKernels/Kernels/Strides.hpp:5-9);
 * the C++ name is an alias of this type. */
typedef struct RocmKernelsStrides {
    int batch;
    int head;
    int token;
} RocmKernelsStrides;

/* Storage type of the generic forward's q, k, v and output, passed as one byte. The values of
 * ROCmKernels::Kernels::DType (ROCmKernels.Kernels/include/ROCmKernels/Kernels/DType.hpp:10,
 * `enum class DType : unsigned char { Float32, Float16 }`); the C++ enum of the same name converts
 * to this type. */
typedef unsigned char RocmKernelsDType;
#define ROCMKERNELS_DTYPE_FLOAT32 ((RocmKernelsDType)0)
#define ROCMKERNELS_DTYPE_FLOAT16 ((RocmKernelsDType)1)

/* cudaStream_t (== hipStream_t through the HIP shim) without requiring the CUDA headers. */
struct CUstream_st;
typedef struct CUstream_st *RocmKernelsStream;

/* 32-wide forward, "simple" entry. Replaces attention_fp32_forward
 * (Attention.hpp:9-11; Attention.hip:194-203). Exact FP32 SIMT kernel. */
ROCMKERNELS_C_EXPORT int attention_fp32_forward(const float *q, const float *k, const float *v, const bool *mask,
        float *output, float *lse, int batch, int heads, int queries, int keys, int radius, RocmKernelsStrides qs,
        RocmKernelsStrides ks, RocmKernelsStrides vs, RocmKernelsStrides os, RocmKernelsStream stream);

/* 32-wide forward, tiled entry. Replaces attention_fp32_forward_tiled
 * (Attention.hpp:12-14; Attention.hip:225-233). */
ROCMKERNELS_C_EXPORT int attention_fp32_forward_tiled(const float *q, const float *k, const float *v, const bool *mask,
        float *output, float *lse, int batch, int heads, int queries, int keys, int radius, RocmKernelsStrides qs,
        RocmKernelsStrides ks, RocmKernelsStrides vs, RocmKernelsStrides os, RocmKernelsStream stream);

/* 32-wide backward: delta = sum(dO * O) per row, then dQ, dK, dV from the saved {max, sum}.
 * Replaces attention_fp32_backward (Attention.hpp:15-18; Attention.hip:205-223). */
ROCMKERNELS_C_EXPORT int attention_fp32_backward(const float *q, const float *k, const float *v, const bool *mask,
        const float *output, const float *lse, const float *upstream, float *gradient_q, float *gradient_k,
        float *gradient_v, float *delta, int batch, int heads, int queries, int keys, int radius, RocmKernelsStrides qs,
        RocmKernelsStrides ks, RocmKernelsStrides vs, RocmKernelsStrides os, RocmKernelsStrides us,
        RocmKernelsStream stream);

/* 32-wide backward, tiled entry. Replaces attention_fp32_backward_tiled
 * (Attention.hpp:19-22; Attention.hip:235-250). */
ROCMKERNELS_C_EXPORT int attention_fp32_backward_tiled(const float *q, const float *k, const float *v, const bool *mask,
        const float *output, const float *lse, const float *upstream, float *gradient_q, float *gradient_k,
        float *gradient_v, float *delta, int batch, int heads, int queries, int keys, int radius, RocmKernelsStrides qs,
        RocmKernelsStrides ks, RocmKernelsStrides vs, RocmKernelsStrides os, RocmKernelsStrides us,
        RocmKernelsStream stream);

/* 32-wide backward in one key-major pass (the single-pass form of attention_fp32_backward, same
 * arguments and outputs plus a workspace): a column pre-pass writes delta, zeroes gradient_q and
 * stores in `workspace` the split-FP16 copies of scaled Q and of upstream and per-64-query
 * statistics; then one kernel computes dK and dV per key and adds each key tile's share of dQ with
 * FP32 atomics, so dQ's summation order over key tiles is not fixed (results may differ in the
 * last bits from run to run; dK, dV and delta are repeatable; the reference's two-kernel split,
 * attention_fp32_backward, is deterministic). `workspace` is device memory of at least
 * attention_fp32_backward_fused_workspace_size(batch, heads, queries) bytes, 128-byte aligned
 * for the single-pass kernels (a null or smaller workspace returns 1; an unaligned one, or
 * tensors the tensor-core kernels cannot address, take the two-pass path); it may be reused
 * between calls that are ordered on one stream. No counterpart in the reference (its backward is
 * the two-pass Attention.hip:205-223). */
ROCMKERNELS_C_EXPORT int attention_fp32_backward_fused(const float *q, const float *k, const float *v, const bool *mask,
        const float *output, const float *lse, const float *upstream, float *gradient_q, float *gradient_k,
        float *gradient_v, float *delta, void *workspace, unsigned long long workspace_bytes, int batch, int heads,
        int queries, int keys, int radius, RocmKernelsStrides qs, RocmKernelsStrides ks, RocmKernelsStrides vs,
        RocmKernelsStrides os, RocmKernelsStrides us, RocmKernelsStream stream);

/* Workspace bytes attention_fp32_backward_fused needs: 256 bytes per query (rounded up to 64
 * queries per (batch, head)) plus 528 bytes per 64 queries; 0 for non-positive sizes. */
ROCMKERNELS_C_EXPORT unsigned long long attention_fp32_backward_fused_workspace_size(int batch, int heads, int queries);

/* Softmax statistics only ({max, sum} per row; no V read, no O write); radius < -1 is invalid.
 * Replaces attention_fp32_statistics (Attention.hpp:23-24; Attention.hip:252-261). */
ROCMKERNELS_C_EXPORT int attention_fp32_statistics(const float *q, const float *k, const bool *mask, float *lse,
        int batch, int heads, int queries, int keys, int radius, RocmKernelsStrides qs, RocmKernelsStrides ks,
        RocmKernelsStream stream);

/* Forward with a tuning selector; group in {2, 4, 8, 84, 164, 1164, 1264}, else error 1.
 * Replaces attention_fp32_forward_tuned (Attention.hpp:25-27; Attention.hip:358-370). */
ROCMKERNELS_C_EXPORT int attention_fp32_forward_tuned(const float *q, const float *k, const float *v, const bool *mask,
        float *output, float *lse, int batch, int heads, int queries, int keys, int radius, int group,
        RocmKernelsStrides qs, RocmKernelsStrides ks, RocmKernelsStrides vs, RocmKernelsStrides os,
        RocmKernelsStream stream);

/* Flash forward, the headline entry: tcgen05/TMEM kernel on sm_100a with split-FP16 operands
 * (kind::f16; each FP32 operand as two FP16 terms, three products) when the tensors are
 * TMA-addressable, else the exact FP32 SIMT kernel; radius < -1 is invalid. Replaces attention_fp32_forward_flash (Attention.hpp:28-30; Attention.hip:372-390).
 * Allocates nothing: the kernel splits each K/V tile itself. */
ROCMKERNELS_C_EXPORT int attention_fp32_forward_flash(const float *q, const float *k, const float *v, const bool *mask,
        float *output, float *lse, int batch, int heads, int queries, int keys, int radius, RocmKernelsStrides qs,
        RocmKernelsStrides ks, RocmKernelsStrides vs, RocmKernelsStrides os, RocmKernelsStream stream);

/* Workspace bytes attention_fp32_forward_flash_workspace needs: 16,400 per 64 keys (rounded up) of
 * each (batch, head); 0 for non-positive sizes. No counterpart in the reference. */
ROCMKERNELS_C_EXPORT unsigned long long attention_fp32_forward_flash_workspace_size(int batch, int heads, int keys);

/* attention_fp32_forward_flash with caller scratch (no counterpart in the reference, whose ABI has
 * no workspace argument): where it pays -- grids beyond one wave of CTAs or key windows of at
 * least 24 tiles of 64 keys -- an operand pre-pass first splits every K/V tile once into
 * `workspace` (the split-FP16 stage images and their headers), and the forward copies them instead
 * of splitting each tile in every CTA; elsewhere, or when `workspace` is not 128-byte aligned, the
 * call runs attention_fp32_forward_flash's kernel. Same results within the same tolerances.
 * `workspace_bytes` below attention_fp32_forward_flash_workspace_size, or a null workspace: error 1.
 * The workspace is in use until the call's work on `stream` completes. */
ROCMKERNELS_C_EXPORT int attention_fp32_forward_flash_workspace(const float *q, const float *k, const float *v,
        const bool *mask, float *output, float *lse, int batch, int heads, int queries, int keys, int radius,
        RocmKernelsStrides qs, RocmKernelsStrides ks, RocmKernelsStrides vs, RocmKernelsStrides os, void *workspace,
        unsigned long long workspace_bytes, RocmKernelsStream stream);

/* Flash forward with a variant selector 0..18, else error 1; radius < -1 is invalid.
 * Replaces attention_fp32_forward_flash_tuned (Attention.hpp:31-33; Attention.hip:392-417). */
ROCMKERNELS_C_EXPORT int attention_fp32_forward_flash_tuned(const float *q, const float *k, const float *v,
        const bool *mask, float *output, float *lse, int batch, int heads, int queries, int keys, int radius,
        int variant, RocmKernelsStrides qs, RocmKernelsStrides ks, RocmKernelsStrides vs, RocmKernelsStrides os,
        RocmKernelsStream stream);

/* Backward with a tuning selector; group in {2, 4, 8, 84, 164, 1164, 1264}, else error 1.
 * Groups 1164 and 1264 compute delta as sum_j P_ij * (dO_i . v_j) (no O read), as the
 * reference's SOFTMAX_DELTA path does. Replaces attention_fp32_backward_tuned
 * (Attention.hpp:34-37; Attention.hip:419-438). */
ROCMKERNELS_C_EXPORT int attention_fp32_backward_tuned(const float *q, const float *k, const float *v, const bool *mask,
        const float *output, const float *lse, const float *upstream, float *gradient_q, float *gradient_k,
        float *gradient_v, float *delta, int batch, int heads, int queries, int keys, int radius, int group,
        RocmKernelsStrides qs, RocmKernelsStrides ks, RocmKernelsStrides vs, RocmKernelsStrides os,
        RocmKernelsStrides us, RocmKernelsStream stream);

/* 64-wide forward. Replaces attention64_fp32_forward (Attention64.hpp:9-11; Attention64.hip:193-202). */
ROCMKERNELS_C_EXPORT int attention64_fp32_forward(const float *q, const float *k, const float *v, const bool *mask,
        float *output, float *lse, int batch, int heads, int queries, int keys, int radius, RocmKernelsStrides qs,
        RocmKernelsStrides ks, RocmKernelsStrides vs, RocmKernelsStrides os, RocmKernelsStream stream);

/* 64-wide backward. Replaces attention64_fp32_backward (Attention64.hpp:12-15; Attention64.hip:204-220). */
ROCMKERNELS_C_EXPORT int attention64_fp32_backward(const float *q, const float *k, const float *v, const bool *mask,
        const float *output, const float *lse, const float *upstream, float *gradient_q, float *gradient_k,
        float *gradient_v, float *delta, int batch, int heads, int queries, int keys, int radius,
        RocmKernelsStrides qs, RocmKernelsStrides ks, RocmKernelsStrides vs, RocmKernelsStrides os,
        RocmKernelsStrides us, RocmKernelsStream stream);

/* Backward split into stages (exported but undeclared in the reference's headers):
 * stage 1 = delta only (softmax-weighted form, no O read), 2 = dQ only (reads delta),
 * 3 = dK/dV only (reads delta). Requires queries >= 32; radius < -1 invalid.
 * Replaces attention_fp32_backward_profile (Attention.hip:327-337). */
ROCMKERNELS_C_EXPORT int attention_fp32_backward_profile(const float *q, const float *k, const float *v,
        const bool *mask, const float *output, const float *lse, const float *upstream, float *gradient_q,
        float *gradient_k, float *gradient_v, float *delta, int batch, int heads, int queries, int keys, int radius,
        int stage, RocmKernelsStrides qs, RocmKernelsStrides ks, RocmKernelsStrides vs, RocmKernelsStrides os,
        RocmKernelsStrides us, RocmKernelsStream stream);

/* dQ stage only (reads delta) with a tuning selector in {14, 18, 24, 28, 44, 116}, else error 1.
 * Requires queries >= 32; radius < -1 invalid. Exported but undeclared in the reference's
 * headers. Replaces attention_fp32_query_profile (Attention.hip:339-356). */
ROCMKERNELS_C_EXPORT int attention_fp32_query_profile(const float *q, const float *k, const float *v,
        const bool *mask, const float *output, const float *lse, const float *upstream, float *gradient_q,
        float *gradient_k, float *gradient_v, float *delta, int batch, int heads, int queries, int keys, int radius,
        int tuning, RocmKernelsStrides qs, RocmKernelsStrides ks, RocmKernelsStrides vs, RocmKernelsStrides os,
        RocmKernelsStrides us, RocmKernelsStream stream);

/* 32-wide backward without a delta argument, for callers that cannot supply or allocate the
 * per-row delta scratch (an interface exposing only dQ/dK/dV, or a step whose device memory is
 * fixed before it runs): the same kernels and results as attention_fp32_backward, with delta kept
 * in a 16 MiB array inside the library, so the call allocates nothing. Limit: batch * heads *
 * queries <= 4194304, else error 1 (cudaErrorInvalidValue). Calls on one device share that
 * array, so they must not overlap (issue them on one stream per device, or order them). The first
 * call on a device looks up the array's device address (cudaGetSymbolAddress) and should come
 * before any stream capture. No counterpart in the reference. */
ROCMKERNELS_C_EXPORT int attention_fp32_backward_static_delta(const float *q, const float *k, const float *v,
        const bool *mask, const float *output, const float *lse, const float *upstream, float *gradient_q,
        float *gradient_k, float *gradient_v, int batch, int heads, int queries, int keys, int radius,
        RocmKernelsStrides qs, RocmKernelsStrides ks, RocmKernelsStrides vs, RocmKernelsStrides os,
        RocmKernelsStrides us, RocmKernelsStream stream);

/* Generic forward for 16-, 32- or 64-wide heads with FP32 or FP16 storage (accumulation FP32),
 * forward only. Replaces attention_generic_forward (Generic/AttentionGeneric.hpp:10-13;
 * AttentionGeneric.hip:292-309): q, k, v and output are `dtype` elements with the given strides
 * (in elements), lse is FP32 {row max, exp sum}. Scores are (q.k) * (1/sqrt(head_width)); a row
 * whose exp sum is not positive (fully masked, or NaN) gives O = 0 and lse = {-inf, 0}, the
 * reference's epilogue (AttentionGeneric.hip:119-128). Returns 1 for null pointers, non-positive
 * sizes, head_width outside {16, 32, 64}, radius < -1 or an unknown dtype.
 * Kernels: FP16 storage runs a tcgen05 kernel with FP16 operands (P rounded to FP16 once, as
 * the reference rounds it for its v_dot2 P.V); FP32 storage with head width 32 or 64 runs the
 * split-FP16 tcgen05 flash kernel; everything else (FP32 with head width 16, or tensors the
 * tensor maps cannot describe) the exact FP32 SIMT kernel. */
ROCMKERNELS_C_EXPORT int attention_generic_forward(const void *q, const void *k, const void *v, const bool *mask,
        void *output, float *lse, int batch, int heads, int queries, int keys, int head_width, int radius,
        RocmKernelsStrides qs, RocmKernelsStrides ks, RocmKernelsStrides vs, RocmKernelsStrides os,
        RocmKernelsDType dtype, RocmKernelsStream stream);

/* Rotary embedding of q and k for 32-wide heads. Replaces rotary_fp32 (Positional/Rotary.hpp:9-11;
 * Rotary.hip:44-56): q, k, cos and sin are read at their strides (the tables' head stride is
 * not used: cos/sin hold 32 values per (batch, token)); oq and ok are written token-major,
 * packed [batch][length][heads][32]. Feature c rotates with feature c + 16:
 * forward lo' = lo cos_lo - hi sin_lo, hi' = hi cos_hi + lo sin_hi; backward != 0 applies the
 * transposed rotation (the gradient). Returns 1 for null pointers or non-positive sizes (and,
 * beyond the reference, for batch * heads * length above 2^29 rows). */
ROCMKERNELS_C_EXPORT int rotary_fp32(const float *q, const float *k, const float *cos, const float *sin, float *oq,
        float *ok, int batch, int heads, int length, int backward, RocmKernelsStrides qs, RocmKernelsStrides ks,
        RocmKernelsStrides cs, RocmKernelsStrides ss, RocmKernelsStream stream);

/* Flash forward with the rotary prologue fused in (no reference counterpart): the result of
 * rotary_fp32 (forward) on q and k followed by attention_fp32_forward_flash on the rotated
 * tensors, bit for bit, without writing or reading the rotated tensors. cos/sin are
 * [batch][token][32] at cs/ss (batch and token strides; rows 0 .. max(queries, keys) - 1 are
 * read: query i and key j use row i and row j). Validation as attention_fp32_forward_flash plus
 * null tables (error 1). Tensor-core kernel when q, k, v are TMA-addressable and the tables
 * 16-byte aligned with strides of 4 floats, else the exact SIMT kernel with the same prologue. */
ROCMKERNELS_C_EXPORT int attention_fp32_forward_flash_rotary(const float *q, const float *k, const float *v,
        const float *cos, const float *sin, const bool *mask, float *output, float *lse, int batch, int heads, int queries,
        int keys, int radius, RocmKernelsStrides qs, RocmKernelsStrides ks, RocmKernelsStrides vs, RocmKernelsStrides cs,
        RocmKernelsStrides ss, RocmKernelsStrides os, RocmKernelsStream stream);

/* attention_fp32_forward_flash_rotary with caller scratch, as attention_fp32_forward_flash_workspace
 * (the pre-pass rotates the K rows as it splits them). No counterpart in the reference. */
ROCMKERNELS_C_EXPORT int attention_fp32_forward_flash_rotary_workspace(const float *q, const float *k, const float *v,
        const float *cos, const float *sin, const bool *mask, float *output, float *lse, int batch, int heads, int queries,
        int keys, int radius, RocmKernelsStrides qs, RocmKernelsStrides ks, RocmKernelsStrides vs, RocmKernelsStrides cs,
        RocmKernelsStrides ss, RocmKernelsStrides os, void *workspace, unsigned long long workspace_bytes,
        RocmKernelsStream stream);

/* Library build identification: a static string naming the architecture the kernels were
 * compiled for ("sm_100a") and the kernel families present. No counterpart in the reference. */
ROCMKERNELS_C_EXPORT const char *rocmkernels_attention_build_info(void);

/* Name of the kernel the flash forward (head_width 32: attention_fp32_forward_flash; 64:
 * attention64_fp32_forward) selects for contiguous, 16-byte aligned tensors of this shape (for
 * benchmarks and profiles). No counterpart in the reference. */
ROCMKERNELS_C_EXPORT const char *rocmkernels_attention_flash_kernel(int batch, int heads, int queries, int keys,
        int head_width);

/* Name of the kernel attention_fp32_forward_flash_workspace selects for contiguous, 16-byte aligned
 * tensors of this shape ("...-prepared" for the operand pre-pass and the forward). No counterpart
 * in the reference. */
ROCMKERNELS_C_EXPORT const char *rocmkernels_attention_flash_workspace_kernel(int batch, int heads, int queries, int keys);

/* Name of the kernel attention_generic_forward runs for contiguous [batch][heads][tokens][head_width]
 * tensors of the given dtype (no reference counterpart; for benchmarks and tests). */
ROCMKERNELS_C_EXPORT const char *rocmkernels_attention_generic_kernel(int batch, int heads, int queries, int keys,
        int head_width, RocmKernelsDType dtype);

/* Status word of the tensor-core kernels on the current device: 0, or 1 when a bounded
 * pipeline wait gave up (a protocol failure; the affected rows are written as NaN). Reading it
 * synchronizes with the device; clear != 0 resets it. No counterpart in the reference. */
ROCMKERNELS_C_EXPORT unsigned int rocmkernels_attention_device_status(int clear);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* ROCMKERNELS_ATTENTION_H */
