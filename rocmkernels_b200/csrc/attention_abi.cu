// The library's extern "C" entry points: argument validation, return codes and dispatch onto the
// sm_100a kernels. Each entry mirrors the launcher of the same name in the reference
// (ROCmKernels.Kernels/src/Attention/Attention.hip:194-438, Attention64.hip:193-220): same
// argument meaning, same validation, same error codes, asynchronous on the caller's stream.
#include <rocmkernels_attention.h>

#include "attention_common.cuh"
#include "attention_simt.cuh"
#include "attention_tc.cuh"

#include <cmath>
#include <mutex>
#include <type_traits>

namespace {

using rk::AttentionParams;

rk::Tensor make_tensor(const float *data, RocmKernelsStrides s) { return rk::Tensor{data, s.batch, s.head, s.token}; }

bool aligned16(const void *pointer) { return (reinterpret_cast<uintptr_t>(pointer) & 15u) == 0; }
bool strides4(RocmKernelsStrides s) { return s.batch % 4 == 0 && s.head % 4 == 0 && s.token % 4 == 0; }

bool forward_args_bad(const float *q, const float *k, const float *v, const bool *mask, const float *output,
                      const float *lse, int batch, int heads, int queries, int keys) {
    return !q || !k || !v || !mask || !output || !lse || batch <= 0 || heads <= 0 || queries <= 0 || keys <= 0;
}

bool backward_args_bad(const float *q, const float *k, const float *v, const bool *mask, const float *output,
                       const float *lse, const float *upstream, const float *gq, const float *gk, const float *gv,
                       const float *delta, int batch, int heads, int queries, int keys) {
    return forward_args_bad(q, k, v, mask, output, lse, batch, heads, queries, keys) || !upstream || !gq || !gk || !gv ||
           !delta;
}

AttentionParams forward_params(int D, const float *q, const float *k, const float *v, const bool *mask, float *output,
                               float *lse, int batch, int heads, int queries, int keys, int radius, RocmKernelsStrides qs,
                               RocmKernelsStrides ks, RocmKernelsStrides vs, RocmKernelsStrides os) {
    AttentionParams p{};
    p.q = make_tensor(q, qs);
    p.k = make_tensor(k, ks);
    p.v = make_tensor(v, vs);
    p.o = rk::OutTensor{output, os.batch, os.head, os.token};
    p.mask = reinterpret_cast<const unsigned char *>(mask);
    p.lse = lse;
    p.batch = batch;
    p.heads = heads;
    p.queries = queries;
    p.keys = keys;
    p.radius = radius;
    p.scale = D == 32 ? 0.17677669529663688f : 0.125f;  // 1/sqrt(D)
    p.vec4 = aligned16(q) && aligned16(k) && (v == nullptr || aligned16(v)) && strides4(qs) && strides4(ks) &&
             (v == nullptr || strides4(vs));
    return p;
}

AttentionParams backward_params(int D, const float *q, const float *k, const float *v, const bool *mask,
                                const float *output, const float *lse, const float *upstream, float *gq, float *gk,
                                float *gv, float *delta, int batch, int heads, int queries, int keys, int radius,
                                RocmKernelsStrides qs, RocmKernelsStrides ks, RocmKernelsStrides vs,
                                RocmKernelsStrides os, RocmKernelsStrides us) {
    AttentionParams p = forward_params(D, q, k, v, mask, nullptr, nullptr, batch, heads, queries, keys, radius, qs, ks, vs, os);
    p.o_in = make_tensor(output, os);
    p.dout = make_tensor(upstream, us);
    p.lse_in = lse;
    p.dq = gq;
    p.dk = gk;
    p.dv = gv;
    p.delta = delta;
    p.vec4 = p.vec4 && aligned16(output) && aligned16(upstream) && strides4(os) && strides4(us);
    return p;
}

unsigned blocks_for(int tokens, int tile, int heads, int batch) {
    return static_cast<unsigned>((tokens + tile - 1) / tile) * static_cast<unsigned>(heads) * static_cast<unsigned>(batch);
}

template <int D, bool STATS_ONLY, class T = float, bool kRotary = false>
int launch_simt_forward(const AttentionParams &p, cudaStream_t stream) {
    constexpr int bytes = rk::simt::ForwardSmem<D, STATS_ONLY>::bytes;
    cudaError_t status = rk::prepare_kernel<rk::simt::forward_kernel<D, STATS_ONLY, T, kRotary>>(bytes);
    if (status != cudaSuccess) return status;
    rk::simt::forward_kernel<D, STATS_ONLY, T, kRotary>
            <<<blocks_for(p.queries, rk::simt::kBlockQ, p.heads, p.batch), rk::simt::kThreads, bytes, stream>>>(p);
    return cudaGetLastError();
}

template <int D, int MODE>
int launch_simt_query(const AttentionParams &p, cudaStream_t stream) {
    constexpr int bytes = rk::simt::QuerySmem<D>::bytes;
    cudaError_t status = rk::prepare_kernel<rk::simt::backward_query_kernel<D, MODE>>(bytes);
    if (status != cudaSuccess) return status;
    rk::simt::backward_query_kernel<D, MODE>
            <<<blocks_for(p.queries, rk::simt::kBlockQ, p.heads, p.batch), rk::simt::kThreads, bytes, stream>>>(p);
    return cudaGetLastError();
}

template <int D>
int launch_simt_key(const AttentionParams &p, cudaStream_t stream) {
    constexpr int bytes = rk::simt::KeySmem<D>::bytes;
    cudaError_t status = rk::prepare_kernel<rk::simt::backward_key_kernel<D>>(bytes);
    if (status != cudaSuccess) return status;
    rk::simt::backward_key_kernel<D>
            <<<blocks_for(p.keys, rk::simt::kBlockK, p.heads, p.batch), rk::simt::kThreads, bytes, stream>>>(p);
    return cudaGetLastError();
}

// Full backward: delta + dQ (query-major), then dK/dV (key-major), ordered on one stream.
// softmax_delta: delta = sum_j P_ij (dO_i . v_j) in its own pass (the reference's SOFTMAX_DELTA
// groups), then dQ reading it.
template <int D>
int launch_backward(const AttentionParams &p, cudaStream_t stream, bool softmax_delta) {
    int status;
    if (softmax_delta) {
        status = launch_simt_query<D, rk::simt::kSoftmaxDelta>(p, stream);
        if (status != cudaSuccess) return status;
        status = launch_simt_query<D, rk::simt::kDqFromDelta>(p, stream);
    } else {
        status = launch_simt_query<D, rk::simt::kDeltaAndDq>(p, stream);
    }
    if (status != cudaSuccess) return status;
    return launch_simt_key<D>(p, stream);
}

// The flash entry: the tcgen05 tensor-core kernel when the problem fits its contract, else the
// exact SIMT kernel (same results within the documented tolerance; no CPU path exists). With a
// workspace the tensor-core kernel may take prepared operands (attention_tc.cuh).
int launch_flash(const AttentionParams &p, void *workspace, cudaStream_t stream) {
    if (rk::tc::flash_supported(p)) {
        const int status = rk::tc::launch_flash_forward(p, 32, workspace, stream);
        if (status != rk::tc::kNotEligible) return status;
    }
    return launch_simt_forward<32, false>(p, stream);
}

// Parameters of the generic forward: T-typed tensors addressed through row_as<T> (strides in
// elements of T), scale 1/sqrt(D) computed as the reference does (AttentionGeneric.hip:245),
// the generic epilogue (NaN totals give 0), 4-element vector loads where every row allows them.
template <class T>
AttentionParams generic_params(int D, const void *q, const void *k, const void *v, const bool *mask, void *output,
                               float *lse, int batch, int heads, int queries, int keys, int radius, RocmKernelsStrides qs,
                               RocmKernelsStrides ks, RocmKernelsStrides vs, RocmKernelsStrides os) {
    AttentionParams p{};
    p.q = make_tensor(static_cast<const float *>(q), qs);
    p.k = make_tensor(static_cast<const float *>(k), ks);
    p.v = make_tensor(static_cast<const float *>(v), vs);
    p.o = rk::OutTensor{static_cast<float *>(output), os.batch, os.head, os.token};
    p.mask = reinterpret_cast<const unsigned char *>(mask);
    p.lse = lse;
    p.batch = batch;
    p.heads = heads;
    p.queries = queries;
    p.keys = keys;
    p.radius = radius;
    p.scale = 1.0f / std::sqrt(static_cast<float>(D));
    p.zero_nan_rows = 1;
    const auto aligned = [](const void *pointer) { return (reinterpret_cast<uintptr_t>(pointer) & (4 * sizeof(T) - 1)) == 0; };
    p.vec4 = aligned(q) && aligned(k) && aligned(v) && strides4(qs) && strides4(ks) && strides4(vs);
    return p;
}

// Generic forward dispatch. FP32 storage: the split-FP16 tensor-core flash kernel (D = 16 on its
// 32-wide form) when its tensor maps describe the tensors, else the exact SIMT kernel.
// FP16 storage: the single-term FP16 tensor-core kernel when K, V and Q rows are 16-byte
// addressable, else the SIMT kernel widening the FP16 values.
template <class T>
int launch_generic(const AttentionParams &p, int D, cudaStream_t stream) {
    if constexpr (std::is_same_v<T, float>) {
        if (rk::tc::flash_supported(p)) {
            const int status = rk::tc::launch_flash_forward(p, D, nullptr, stream);
            if (status != rk::tc::kNotEligible) return status;
        }
    } else {
        if (rk::tc::half_flash_supported(p)) {
            const int status = rk::tc::launch_half_flash_forward(p, D, stream);
            if (status != rk::tc::kNotEligible) return status;
        }
    }
    if (D == 16) return launch_simt_forward<16, false, T>(p, stream);
    if (D == 32) return launch_simt_forward<32, false, T>(p, stream);
    return launch_simt_forward<64, false, T>(p, stream);
}

bool known_group(int group) {
    return group == 2 || group == 4 || group == 8 || group == 84 || group == 164 || group == 1164 || group == 1264;
}

// Delta scratch for attention_fp32_backward_static_delta. Some callers cannot hand the backward
// a delta buffer: an autograd interface that exposes only dQ, dK and dV, or a training step whose
// device memory is planned up front and must not grow once it runs. For them the per-row delta
// lives in this file-scope array of the library instead of caller memory, so the call allocates
// nothing. Nothing in it has to start at zero: the query-major pass writes every entry it covers
// before the key-major pass reads it. Calls on one device share it, so they must not overlap.
constexpr long long kStaticDeltaRows = 1ll << 22;  // batch * heads * queries <= 4,194,304 (16 MiB)
static __device__ __align__(256) float g_static_delta[kStaticDeltaRows];

// Device address of g_static_delta on the current device, looked up (with that device current)
// by the first call in each context. The address belongs to the context: cudaDeviceReset
// (ROCmKernels::ResetDevice, or anyone else in the process) unloads the module that holds the
// array, and the context the runtime creates next may place it elsewhere, so each entry records
// the context key it was taken in and is looked up again when another context is current.
cudaError_t static_delta_address(float **address) {
    constexpr int kDevices = 64;
    static std::mutex lock;
    static float *addresses[kDevices] = {};
    static unsigned long long keys[kDevices] = {};
    int device = 0;
    cudaError_t status = cudaGetDevice(&device);
    if (status != cudaSuccess) return status;
    if (device < 0 || device >= kDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> guard(lock);
    const unsigned long long key = rk::context_key();
    if (key == 0 || keys[device] != key || addresses[device] == nullptr) {
        void *pointer = nullptr;
        status = cudaGetSymbolAddress(&pointer, g_static_delta);  // creates the context if needed
        if (status != cudaSuccess) return status;
        addresses[device] = static_cast<float *>(pointer);
        keys[device] = rk::context_key();
    }
    *address = addresses[device];
    return cudaSuccess;
}

}  // namespace

extern "C" {

int attention_fp32_forward(const float *q, const float *k, const float *v, const bool *mask, float *output, float *lse,
                           int batch, int heads, int queries, int keys, int radius, RocmKernelsStrides qs,
                           RocmKernelsStrides ks, RocmKernelsStrides vs, RocmKernelsStrides os, RocmKernelsStream stream) {
    if (forward_args_bad(q, k, v, mask, output, lse, batch, heads, queries, keys)) return cudaErrorInvalidValue;
    const AttentionParams p = forward_params(32, q, k, v, mask, output, lse, batch, heads, queries, keys, radius, qs, ks, vs, os);
    return launch_simt_forward<32, false>(p, stream);
}

int attention_fp32_forward_tiled(const float *q, const float *k, const float *v, const bool *mask, float *output,
                                 float *lse, int batch, int heads, int queries, int keys, int radius,
                                 RocmKernelsStrides qs, RocmKernelsStrides ks, RocmKernelsStrides vs,
                                 RocmKernelsStrides os, RocmKernelsStream stream) {
    return attention_fp32_forward(q, k, v, mask, output, lse, batch, heads, queries, keys, radius, qs, ks, vs, os, stream);
}

int attention_fp32_backward(const float *q, const float *k, const float *v, const bool *mask, const float *output,
                            const float *lse, const float *upstream, float *gradient_q, float *gradient_k,
                            float *gradient_v, float *delta, int batch, int heads, int queries, int keys, int radius,
                            RocmKernelsStrides qs, RocmKernelsStrides ks, RocmKernelsStrides vs, RocmKernelsStrides os,
                            RocmKernelsStrides us, RocmKernelsStream stream) {
    if (backward_args_bad(q, k, v, mask, output, lse, upstream, gradient_q, gradient_k, gradient_v, delta, batch, heads,
                          queries, keys))
        return cudaErrorInvalidValue;
    const AttentionParams p = backward_params(32, q, k, v, mask, output, lse, upstream, gradient_q, gradient_k, gradient_v,
                                              delta, batch, heads, queries, keys, radius, qs, ks, vs, os, us);
    // The tensor-core backward when the tensors are TMA-addressable, else the exact SIMT pair
    // (which the tuned entry always runs, so both stay reachable).
    if (rk::tc::backward_supported(p)) {
        const int status = rk::tc::launch_backward(p, 32, stream);
        if (status != rk::tc::kNotEligible) return status;
    }
    return launch_backward<32>(p, stream, false);
}

unsigned long long attention_fp32_backward_fused_workspace_size(int batch, int heads, int queries) {
    if (batch <= 0 || heads <= 0 || queries <= 0) return 0;
    return static_cast<unsigned long long>(
            rk::tc::fused_backward_workspace_bytes(static_cast<long long>(batch) * heads, queries));
}

int attention_fp32_backward_fused(const float *q, const float *k, const float *v, const bool *mask, const float *output,
                                  const float *lse, const float *upstream, float *gradient_q, float *gradient_k,
                                  float *gradient_v, float *delta, void *workspace, unsigned long long workspace_bytes,
                                  int batch, int heads, int queries, int keys, int radius, RocmKernelsStrides qs,
                                  RocmKernelsStrides ks, RocmKernelsStrides vs, RocmKernelsStrides os, RocmKernelsStrides us,
                                  RocmKernelsStream stream) {
    if (backward_args_bad(q, k, v, mask, output, lse, upstream, gradient_q, gradient_k, gradient_v, delta, batch, heads,
                          queries, keys) ||
        !workspace || workspace_bytes < attention_fp32_backward_fused_workspace_size(batch, heads, queries))
        return cudaErrorInvalidValue;
    const AttentionParams p = backward_params(32, q, k, v, mask, output, lse, upstream, gradient_q, gradient_k, gradient_v,
                                              delta, batch, heads, queries, keys, radius, qs, ks, vs, os, us);
    // Tensors the tensor maps cannot describe (or a workspace that is not 128-byte aligned) take
    // the two-pass backward: the same results up to the order of dQ's sums.
    if (rk::tc::backward_supported(p)) {
        const int status = rk::tc::launch_fused_backward(p, workspace, stream);
        if (status != rk::tc::kNotEligible) return status;
    }
    return attention_fp32_backward(q, k, v, mask, output, lse, upstream, gradient_q, gradient_k, gradient_v, delta, batch,
                                   heads, queries, keys, radius, qs, ks, vs, os, us, stream);
}

int attention_fp32_backward_tiled(const float *q, const float *k, const float *v, const bool *mask,
                                  const float *output, const float *lse, const float *upstream, float *gradient_q,
                                  float *gradient_k, float *gradient_v, float *delta, int batch, int heads, int queries,
                                  int keys, int radius, RocmKernelsStrides qs, RocmKernelsStrides ks,
                                  RocmKernelsStrides vs, RocmKernelsStrides os, RocmKernelsStrides us,
                                  RocmKernelsStream stream) {
    return attention_fp32_backward(q, k, v, mask, output, lse, upstream, gradient_q, gradient_k, gradient_v, delta, batch,
                                   heads, queries, keys, radius, qs, ks, vs, os, us, stream);
}

int attention_fp32_statistics(const float *q, const float *k, const bool *mask, float *lse, int batch, int heads,
                              int queries, int keys, int radius, RocmKernelsStrides qs, RocmKernelsStrides ks,
                              RocmKernelsStream stream) {
    if (!q || !k || !mask || !lse || batch <= 0 || heads <= 0 || queries <= 0 || keys <= 0 || radius < -1)
        return cudaErrorInvalidValue;
    const AttentionParams p =
            forward_params(32, q, k, nullptr, mask, nullptr, lse, batch, heads, queries, keys, radius, qs, ks, ks, ks);
    if (rk::tc::statistics_supported(p)) {
        const int status = rk::tc::launch_statistics(p, stream);
        if (status != rk::tc::kNotEligible) return status;
    }
    return launch_simt_forward<32, true>(p, stream);
}

int attention_fp32_forward_tuned(const float *q, const float *k, const float *v, const bool *mask, float *output,
                                 float *lse, int batch, int heads, int queries, int keys, int radius, int group,
                                 RocmKernelsStrides qs, RocmKernelsStrides ks, RocmKernelsStrides vs,
                                 RocmKernelsStrides os, RocmKernelsStream stream) {
    if (!known_group(group)) return cudaErrorInvalidValue;
    return attention_fp32_forward(q, k, v, mask, output, lse, batch, heads, queries, keys, radius, qs, ks, vs, os, stream);
}

int attention_fp32_forward_flash(const float *q, const float *k, const float *v, const bool *mask, float *output,
                                 float *lse, int batch, int heads, int queries, int keys, int radius,
                                 RocmKernelsStrides qs, RocmKernelsStrides ks, RocmKernelsStrides vs,
                                 RocmKernelsStrides os, RocmKernelsStream stream) {
    if (forward_args_bad(q, k, v, mask, output, lse, batch, heads, queries, keys) || radius < -1)
        return cudaErrorInvalidValue;
    const AttentionParams p = forward_params(32, q, k, v, mask, output, lse, batch, heads, queries, keys, radius, qs, ks, vs, os);
    return launch_flash(p, nullptr, stream);
}

unsigned long long attention_fp32_forward_flash_workspace_size(int batch, int heads, int keys) {
    if (batch <= 0 || heads <= 0 || keys <= 0) return 0;
    return static_cast<unsigned long long>(rk::tc::prepared_forward_bytes(batch, heads, keys));
}

int attention_fp32_forward_flash_workspace(const float *q, const float *k, const float *v, const bool *mask, float *output,
                                           float *lse, int batch, int heads, int queries, int keys, int radius,
                                           RocmKernelsStrides qs, RocmKernelsStrides ks, RocmKernelsStrides vs,
                                           RocmKernelsStrides os, void *workspace, unsigned long long workspace_bytes,
                                           RocmKernelsStream stream) {
    if (forward_args_bad(q, k, v, mask, output, lse, batch, heads, queries, keys) || radius < -1 || !workspace ||
        workspace_bytes < attention_fp32_forward_flash_workspace_size(batch, heads, keys))
        return cudaErrorInvalidValue;
    const AttentionParams p = forward_params(32, q, k, v, mask, output, lse, batch, heads, queries, keys, radius, qs, ks, vs, os);
    return launch_flash(p, workspace, stream);
}

int attention_fp32_forward_flash_tuned(const float *q, const float *k, const float *v, const bool *mask, float *output,
                                       float *lse, int batch, int heads, int queries, int keys, int radius, int variant,
                                       RocmKernelsStrides qs, RocmKernelsStrides ks, RocmKernelsStrides vs,
                                       RocmKernelsStrides os, RocmKernelsStream stream) {
    if (variant < 0 || variant > 18) return cudaErrorInvalidValue;
    if (forward_args_bad(q, k, v, mask, output, lse, batch, heads, queries, keys) || radius < -1)
        return cudaErrorInvalidValue;
    const AttentionParams p = forward_params(32, q, k, v, mask, output, lse, batch, heads, queries, keys, radius, qs, ks, vs, os);
    // Variants 0-18 were the reference's register/LDS tiling sweep; on sm_100a the even
    // variants run the tensor-core kernel and the odd ones the exact SIMT kernel, so both
    // implementations stay reachable through the reference's selector.
    if (variant % 2 == 0 || variant == 13) return launch_flash(p, nullptr, stream);
    return launch_simt_forward<32, false>(p, stream);
}

int attention_fp32_backward_tuned(const float *q, const float *k, const float *v, const bool *mask, const float *output,
                                  const float *lse, const float *upstream, float *gradient_q, float *gradient_k,
                                  float *gradient_v, float *delta, int batch, int heads, int queries, int keys,
                                  int radius, int group, RocmKernelsStrides qs, RocmKernelsStrides ks,
                                  RocmKernelsStrides vs, RocmKernelsStrides os, RocmKernelsStrides us,
                                  RocmKernelsStream stream) {
    if (!known_group(group)) return cudaErrorInvalidValue;
    if (backward_args_bad(q, k, v, mask, output, lse, upstream, gradient_q, gradient_k, gradient_v, delta, batch, heads,
                          queries, keys))
        return cudaErrorInvalidValue;
    const AttentionParams p = backward_params(32, q, k, v, mask, output, lse, upstream, gradient_q, gradient_k, gradient_v,
                                              delta, batch, heads, queries, keys, radius, qs, ks, vs, os, us);
    return launch_backward<32>(p, stream, group == 1164 || group == 1264);
}

int attention64_fp32_forward(const float *q, const float *k, const float *v, const bool *mask, float *output, float *lse,
                             int batch, int heads, int queries, int keys, int radius, RocmKernelsStrides qs,
                             RocmKernelsStrides ks, RocmKernelsStrides vs, RocmKernelsStrides os,
                             RocmKernelsStream stream) {
    if (forward_args_bad(q, k, v, mask, output, lse, batch, heads, queries, keys)) return cudaErrorInvalidValue;
    const AttentionParams p = forward_params(64, q, k, v, mask, output, lse, batch, heads, queries, keys, radius, qs, ks, vs, os);
    if (rk::tc::flash_supported(p)) {  // else (tensors not TMA-addressable) the exact SIMT kernel
        const int status = rk::tc::launch_flash_forward(p, 64, nullptr, stream);
        if (status != rk::tc::kNotEligible) return status;
    }
    return launch_simt_forward<64, false>(p, stream);
}

int attention64_fp32_backward(const float *q, const float *k, const float *v, const bool *mask, const float *output,
                              const float *lse, const float *upstream, float *gradient_q, float *gradient_k,
                              float *gradient_v, float *delta, int batch, int heads, int queries, int keys, int radius,
                              RocmKernelsStrides qs, RocmKernelsStrides ks, RocmKernelsStrides vs,
                              RocmKernelsStrides os, RocmKernelsStrides us, RocmKernelsStream stream) {
    if (backward_args_bad(q, k, v, mask, output, lse, upstream, gradient_q, gradient_k, gradient_v, delta, batch, heads,
                          queries, keys))
        return cudaErrorInvalidValue;
    const AttentionParams p = backward_params(64, q, k, v, mask, output, lse, upstream, gradient_q, gradient_k, gradient_v,
                                              delta, batch, heads, queries, keys, radius, qs, ks, vs, os, us);
    if (rk::tc::backward_supported(p)) {  // else (strides not TMA-addressable) the exact SIMT pair
        const int status = rk::tc::launch_backward(p, 64, stream);
        if (status != rk::tc::kNotEligible) return status;
    }
    return launch_backward<64>(p, stream, false);
}

int attention_fp32_backward_profile(const float *q, const float *k, const float *v, const bool *mask,
                                    const float *output, const float *lse, const float *upstream, float *gradient_q,
                                    float *gradient_k, float *gradient_v, float *delta, int batch, int heads,
                                    int queries, int keys, int radius, int stage, RocmKernelsStrides qs,
                                    RocmKernelsStrides ks, RocmKernelsStrides vs, RocmKernelsStrides os,
                                    RocmKernelsStrides us, RocmKernelsStream stream) {
    if (stage < 1 || stage > 3 || queries < 32 || radius < -1 ||
        backward_args_bad(q, k, v, mask, output, lse, upstream, gradient_q, gradient_k, gradient_v, delta, batch, heads,
                          queries, keys))
        return cudaErrorInvalidValue;
    const AttentionParams p = backward_params(32, q, k, v, mask, output, lse, upstream, gradient_q, gradient_k, gradient_v,
                                              delta, batch, heads, queries, keys, radius, qs, ks, vs, os, us);
    if (stage == 1) return launch_simt_query<32, rk::simt::kSoftmaxDelta>(p, stream);
    if (stage == 2) return launch_simt_query<32, rk::simt::kDqFromDelta>(p, stream);
    return launch_simt_key<32>(p, stream);
}

int attention_fp32_query_profile(const float *q, const float *k, const float *v, const bool *mask, const float *output,
                                 const float *lse, const float *upstream, float *gradient_q, float *gradient_k,
                                 float *gradient_v, float *delta, int batch, int heads, int queries, int keys,
                                 int radius, int tuning, RocmKernelsStrides qs, RocmKernelsStrides ks,
                                 RocmKernelsStrides vs, RocmKernelsStrides os, RocmKernelsStrides us,
                                 RocmKernelsStream stream) {
    if (queries < 32 || radius < -1 ||
        backward_args_bad(q, k, v, mask, output, lse, upstream, gradient_q, gradient_k, gradient_v, delta, batch, heads,
                          queries, keys))
        return cudaErrorInvalidValue;
    if (tuning != 14 && tuning != 18 && tuning != 116 && tuning != 24 && tuning != 28 && tuning != 44)
        return cudaErrorInvalidValue;
    const AttentionParams p = backward_params(32, q, k, v, mask, output, lse, upstream, gradient_q, gradient_k, gradient_v,
                                              delta, batch, heads, queries, keys, radius, qs, ks, vs, os, us);
    return launch_simt_query<32, rk::simt::kDqFromDelta>(p, stream);
}

const char *rocmkernels_attention_build_info(void) { return rk::tc::build_info(); }

unsigned int rocmkernels_attention_device_status(int clear) {
    return rk::tc::read_device_status(clear != 0) | rk::tc::read_backward_status(clear != 0);
}

namespace {
const char *flash_kernel_of(int batch, int heads, int queries, int keys, int head_width, bool workspace) {
    if (head_width != 32 && head_width != 64) return "unsupported";
    AttentionParams p{};
    p.batch = batch;
    p.heads = heads;
    p.queries = queries;
    p.keys = keys;
    p.radius = -1;
    p.vec4 = 1;
    const long long w = head_width;
    p.q = rk::Tensor{nullptr, (long long)heads * queries * w, (long long)queries * w, w};
    p.k = rk::Tensor{nullptr, (long long)heads * keys * w, (long long)keys * w, w};
    p.v = p.k;
    p.o = rk::OutTensor{nullptr, p.q.sb, p.q.sh, p.q.st};
    if (rk::tc::flash_supported(p)) return rk::tc::kernel_name(p, head_width, workspace);
    return head_width == 64 ? "simt-fp32-forward-d64" : "simt-fp32-forward-d32";
}
}  // namespace

const char *rocmkernels_attention_flash_kernel(int batch, int heads, int queries, int keys, int head_width) {
    return flash_kernel_of(batch, heads, queries, keys, head_width, false);
}

const char *rocmkernels_attention_flash_workspace_kernel(int batch, int heads, int queries, int keys) {
    return flash_kernel_of(batch, heads, queries, keys, 32, true);
}

namespace {
int flash_rotary(const float *q, const float *k, const float *v, const float *cos, const float *sin, const bool *mask, float *output,
                 float *lse, int batch, int heads, int queries, int keys, int radius, RocmKernelsStrides qs, RocmKernelsStrides ks,
                 RocmKernelsStrides vs, RocmKernelsStrides cs, RocmKernelsStrides ss, RocmKernelsStrides os, void *workspace,
                 RocmKernelsStream stream) {
    AttentionParams p = forward_params(32, q, k, v, mask, output, lse, batch, heads, queries, keys, radius, qs, ks, vs, os);
    p.rot_cos = cos;
    p.rot_sin = sin;
    p.rot_cb = cs.batch;
    p.rot_ct = cs.token;
    p.rot_sb = ss.batch;
    p.rot_st = ss.token;
    if (rk::tc::flash_supported(p)) {  // else (tensors or tables not 16-byte addressable) the exact SIMT kernel
        const int status = rk::tc::launch_flash_forward_rotary(p, workspace, stream);
        if (status != rk::tc::kNotEligible) return status;
    }
    return launch_simt_forward<32, false, float, true>(p, stream);
}
}  // namespace

int attention_fp32_forward_flash_rotary(const float *q, const float *k, const float *v, const float *cos, const float *sin,
                                        const bool *mask, float *output, float *lse, int batch, int heads, int queries,
                                        int keys, int radius, RocmKernelsStrides qs, RocmKernelsStrides ks,
                                        RocmKernelsStrides vs, RocmKernelsStrides cs, RocmKernelsStrides ss,
                                        RocmKernelsStrides os, RocmKernelsStream stream) {
    if (forward_args_bad(q, k, v, mask, output, lse, batch, heads, queries, keys) || !cos || !sin || radius < -1)
        return cudaErrorInvalidValue;
    return flash_rotary(q, k, v, cos, sin, mask, output, lse, batch, heads, queries, keys, radius, qs, ks, vs, cs, ss, os, nullptr,
                        stream);
}

int attention_fp32_forward_flash_rotary_workspace(const float *q, const float *k, const float *v, const float *cos,
                                                  const float *sin, const bool *mask, float *output, float *lse, int batch,
                                                  int heads, int queries, int keys, int radius, RocmKernelsStrides qs,
                                                  RocmKernelsStrides ks, RocmKernelsStrides vs, RocmKernelsStrides cs,
                                                  RocmKernelsStrides ss, RocmKernelsStrides os, void *workspace,
                                                  unsigned long long workspace_bytes, RocmKernelsStream stream) {
    if (forward_args_bad(q, k, v, mask, output, lse, batch, heads, queries, keys) || !cos || !sin || radius < -1 || !workspace ||
        workspace_bytes < attention_fp32_forward_flash_workspace_size(batch, heads, keys))
        return cudaErrorInvalidValue;
    return flash_rotary(q, k, v, cos, sin, mask, output, lse, batch, heads, queries, keys, radius, qs, ks, vs, cs, ss, os, workspace,
                        stream);
}

int attention_generic_forward(const void *q, const void *k, const void *v, const bool *mask, void *output, float *lse,
                              int batch, int heads, int queries, int keys, int head_width, int radius, RocmKernelsStrides qs,
                              RocmKernelsStrides ks, RocmKernelsStrides vs, RocmKernelsStrides os, RocmKernelsDType dtype,
                              RocmKernelsStream stream) {
    if (!q || !k || !v || !mask || !output || !lse || batch <= 0 || heads <= 0 || queries <= 0 || keys <= 0)
        return cudaErrorInvalidValue;
    if (head_width != 16 && head_width != 32 && head_width != 64) return cudaErrorInvalidValue;
    if (radius < -1) return cudaErrorInvalidValue;
    if (dtype == ROCMKERNELS_DTYPE_FLOAT32) {
        const AttentionParams p = generic_params<float>(head_width, q, k, v, mask, output, lse, batch, heads, queries, keys,
                                                        radius, qs, ks, vs, os);
        return launch_generic<float>(p, head_width, stream);
    }
    if (dtype == ROCMKERNELS_DTYPE_FLOAT16) {
        const AttentionParams p = generic_params<__half>(head_width, q, k, v, mask, output, lse, batch, heads, queries, keys,
                                                         radius, qs, ks, vs, os);
        return launch_generic<__half>(p, head_width, stream);
    }
    return cudaErrorInvalidValue;
}

const char *rocmkernels_attention_generic_kernel(int batch, int heads, int queries, int keys, int head_width,
                                                 RocmKernelsDType dtype) {
    if ((head_width != 16 && head_width != 32 && head_width != 64) ||
        (dtype != ROCMKERNELS_DTYPE_FLOAT32 && dtype != ROCMKERNELS_DTYPE_FLOAT16))
        return "unsupported";
    const bool half = dtype == ROCMKERNELS_DTYPE_FLOAT16;
    const long long w = head_width;
    AttentionParams p{};
    p.batch = batch;
    p.heads = heads;
    p.queries = queries;
    p.keys = keys;
    p.radius = -1;
    p.vec4 = 1;
    p.q = rk::Tensor{nullptr, (long long)heads * queries * w, (long long)queries * w, w};
    p.k = rk::Tensor{nullptr, (long long)heads * keys * w, (long long)keys * w, w};
    p.v = p.k;
    p.o = rk::OutTensor{nullptr, p.q.sb, p.q.sh, p.q.st};
    // A 256-byte aligned stand-in address: the tensor-map check reads no memory.
    p.q.data = p.k.data = p.v.data = reinterpret_cast<const float *>(uintptr_t{1} << 20);
    p.o.data = reinterpret_cast<float *>(uintptr_t{1} << 20);
    if (half && rk::tc::half_flash_supported(p) && rk::tc::tensor_maps_encodable(p, head_width, true))
        return rk::tc::half_kernel_name(head_width);
    if (!half && rk::tc::flash_supported(p) && rk::tc::tensor_maps_encodable(p, head_width, false))
        return rk::tc::kernel_name(p, head_width, false);
    if (half) return head_width == 16 ? "simt-fp16-forward-d16" : head_width == 32 ? "simt-fp16-forward-d32" : "simt-fp16-forward-d64";
    return head_width == 16 ? "simt-fp32-forward-d16" : head_width == 32 ? "simt-fp32-forward-d32" : "simt-fp32-forward-d64";
}

int attention_fp32_backward_static_delta(const float *q, const float *k, const float *v, const bool *mask,
                                         const float *output, const float *lse, const float *upstream, float *gradient_q,
                                         float *gradient_k, float *gradient_v, int batch, int heads, int queries, int keys,
                                         int radius, RocmKernelsStrides qs, RocmKernelsStrides ks, RocmKernelsStrides vs,
                                         RocmKernelsStrides os, RocmKernelsStrides us, RocmKernelsStream stream) {
    if (batch > 0 && heads > 0 && queries > 0 &&
        static_cast<long long>(batch) * heads * queries > kStaticDeltaRows)
        return cudaErrorInvalidValue;
    float *delta = nullptr;
    const cudaError_t status = static_delta_address(&delta);
    if (status != cudaSuccess) return status;
    return attention_fp32_backward(q, k, v, mask, output, lse, upstream, gradient_q, gradient_k, gradient_v, delta, batch,
                                   heads, queries, keys, radius, qs, ks, vs, os, us, stream);
}

}  // extern "C"
