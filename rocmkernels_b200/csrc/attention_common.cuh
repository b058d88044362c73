// Shared device helpers and launch parameters for the FP32 attention kernels (sm_100a).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "context.h"

namespace rk {

constexpr float kLog2e = 1.4426950408889634f;

// A strided [batch][head][token][feature] tensor; feature stride is 1.
// Element (b, h, t, c) is data[b*sb + h*sh + t*st + c], the addressing of the reference's
// Input::read (Attention.hip:14-20), evaluated in 64-bit here. The strides count elements of the
// storage type: FP32 everywhere except the FP16 tensors of the generic forward, which read them
// through row_as<__half>.
struct Tensor {
    const float *data;
    long long sb, sh, st;
    __device__ __forceinline__ const float *row(int b, int h, int t) const { return row_as<float>(b, h, t); }
    template <class T>
    __device__ __forceinline__ const T *row_as(int b, int h, int t) const {
        return reinterpret_cast<const T *>(data) + (long long)b * sb + (long long)h * sh + (long long)t * st;
    }
};

struct OutTensor {
    float *data;
    long long sb, sh, st;
    __device__ __forceinline__ float *row(int b, int h, int t) const { return row_as<float>(b, h, t); }
    template <class T>
    __device__ __forceinline__ T *row_as(int b, int h, int t) const {
        return reinterpret_cast<T *>(data) + (long long)b * sb + (long long)h * sh + (long long)t * st;
    }
};

// Everything a forward or backward launch needs. Packed outputs (lse, delta, gradients) are
// indexed by the flattened row (b*heads + h)*tokens + t.
struct AttentionParams {
    Tensor q, k, v, o_in, dout;
    OutTensor o;
    const unsigned char *mask;  // [batch][keys], nonzero = visible
    float *lse;                 // [batch][heads][queries][2]
    float *delta;               // [batch][heads][queries]
    float *dq, *dk, *dv;        // packed [batch][heads][tokens][D]
    const float *lse_in;        // saved statistics for the backward
    int batch, heads, queries, keys, radius;
    float scale;                // 1/sqrt(D)
    int vec4;                   // every strided row starts 4-element aligned (float4 / 4 x FP16 loads)
    int zero_nan_rows;          // a row whose exponent sum is NaN gives O = 0 and {-inf, 0} (the generic
                                // forward's epilogue, AttentionGeneric.hip:119-128) instead of NaN
    // Rotary prologue (forward kernels built with it): q and k rows are rotated by the tables of
    // their (batch, token) before use; tables [batch][token][32] at these element strides.
    const float *rot_cos, *rot_sin;
    long long rot_cb, rot_ct, rot_sb, rot_st;
    __device__ __forceinline__ const float *cos_row(int b, int t) const { return rot_cos + b * rot_cb + t * rot_ct; }
    __device__ __forceinline__ const float *sin_row(int b, int t) const { return rot_sin + b * rot_sb + t * rot_st; }
};

// Four consecutive elements widened to FP32: one 16-byte load for FP32, one 8-byte load for FP16.
__device__ __forceinline__ float4 load4(const float *src) { return __ldg(reinterpret_cast<const float4 *>(src)); }
__device__ __forceinline__ float4 load4(const __half *src) {
    const uint2 raw = __ldg(reinterpret_cast<const uint2 *>(src));
    const float2 lo = __half22float2(*reinterpret_cast<const __half2 *>(&raw.x));
    const float2 hi = __half22float2(*reinterpret_cast<const __half2 *>(&raw.y));
    return make_float4(lo.x, lo.y, hi.x, hi.y);
}
__device__ __forceinline__ float load1(const float *src) { return __ldg(src); }
__device__ __forceinline__ float load1(const __half *src) { return __half2float(__ldg(src)); }
__device__ __forceinline__ void store1(float *dst, float value) { *dst = value; }
__device__ __forceinline__ void store1(__half *dst, float value) { *dst = __float2half_rn(value); }

// 2^x on the MUFU unit (PTX ex2.approx.ftz.f32; relative error about 2^-22).
__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Visibility of key j for query i: the selection rule of the reference
// (AttentionFlash32.h:87-94; AttentionTests.cpp:54-59).
__device__ __forceinline__ bool in_window(int query, int key, int radius) {
    return radius < 0 || abs(query - key) <= radius;
}

// Key range [first, last) that can be visible from the query block [q0, q1).
__host__ __device__ __forceinline__ void key_window(int q0, int q1, int keys, int radius, int &first, int &last) {
    first = radius < 0 ? 0 : max(0, q0 - radius);
    last = radius < 0 ? keys : min(keys, q1 + radius);
}

// Configures the dynamic shared memory limit of a kernel once per device and context: the
// attribute belongs to the context, so a device reset (which destroys it) makes the next launch
// set it again (context.h).
template <auto KernelFn>
inline cudaError_t prepare_kernel(int shared_bytes) {
    constexpr int kDevices = 64;
    static std::atomic<unsigned long long> configured[kDevices] = {};
    int device = 0;
    cudaError_t status = cudaGetDevice(&device);
    if (status != cudaSuccess) return status;
    const int slot = device & (kDevices - 1);
    const unsigned long long key = context_key();
    if (key != 0 && configured[slot].load(std::memory_order_acquire) == key) return cudaSuccess;
    status = cudaFuncSetAttribute(KernelFn, cudaFuncAttributeMaxDynamicSharedMemorySize, shared_bytes);
    if (status == cudaSuccess) configured[slot].store(context_key(), std::memory_order_release);
    return status;
}

}  // namespace rk
