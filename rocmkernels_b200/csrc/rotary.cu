// rotary_fp32 (Rotary.hpp:9-11, Rotary.hip:44-56): rotary embedding of q and k for 32-wide heads,
// written token-major ([batch][length][heads][32]) whatever the input strides.
//
// HBM-bound elementwise work (read q, k and the two tables, write oq, ok): one thread per
// (batch, token, head, quarter) handles four low features and their four high partners of both
// q and k, with 16-byte loads and stores where every row allows them. Consecutive threads walk
// the quarters, then the heads, so a warp writes 1 KB of contiguous output; the tables of a
// (batch, token) are read once per head from L1/L2.
#include <rocmkernels_attention.h>

#include "rotary.cuh"

#include <climits>
#include <cstdint>

namespace {

struct RotaryArgs {
    const float *q, *k, *cos, *sin;
    float *oq, *ok;
    long long qb, qh, qt, kb, kh, kt, cb, ct, sb, st;  // element strides (the tables have no head stride)
    int heads, length;
    unsigned rows;  // batch * length * heads
};

template <bool kVec>
__device__ __forceinline__ void load_chunk(const float *p, float (&x)[4]) {
    if constexpr (kVec) {
        const float4 v = __ldg(reinterpret_cast<const float4 *>(p));
        x[0] = v.x, x[1] = v.y, x[2] = v.z, x[3] = v.w;
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) x[i] = __ldg(p + i);
    }
}

template <bool kVec>
__device__ __forceinline__ void store_chunk(float *p, const float (&x)[4]) {
    if constexpr (kVec) {
        *reinterpret_cast<float4 *>(p) = make_float4(x[0], x[1], x[2], x[3]);
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) p[i] = x[i];
    }
}

template <bool kBackward, bool kVec>
__global__ void __launch_bounds__(256) rotary_kernel(const RotaryArgs a) {
    const unsigned item = blockIdx.x * blockDim.x + threadIdx.x;
    const unsigned row = item >> 2;
    if (row >= a.rows) return;
    const int c = 4 * (item & 3);
    const int head = row % a.heads;
    const unsigned bt = row / a.heads;  // batch * length + token
    const int token = bt % a.length;
    const int b = bt / a.length;

    float cl[4], ch[4], sl[4], sh[4];
    const float *cos_row = a.cos + b * a.cb + token * a.ct;
    const float *sin_row = a.sin + b * a.sb + token * a.st;
    load_chunk<kVec>(cos_row + c, cl);
    load_chunk<kVec>(cos_row + c + 16, ch);
    load_chunk<kVec>(sin_row + c, sl);
    load_chunk<kVec>(sin_row + c + 16, sh);

    const long long out_offset = static_cast<long long>(row) * 32 + c;
#pragma unroll
    for (int tensor = 0; tensor < 2; ++tensor) {
        const float *x = tensor == 0 ? a.q + b * a.qb + head * a.qh + token * a.qt : a.k + b * a.kb + head * a.kh + token * a.kt;
        float lo[4], hi[4], out_lo[4], out_hi[4];
        load_chunk<kVec>(x + c, lo);
        load_chunk<kVec>(x + c + 16, hi);
#pragma unroll
        for (int i = 0; i < 4; ++i) rk::rotate_pair<kBackward>(lo[i], hi[i], cl[i], ch[i], sl[i], sh[i], out_lo[i], out_hi[i]);
        float *out = (tensor == 0 ? a.oq : a.ok) + out_offset;
        store_chunk<kVec>(out, out_lo);
        store_chunk<kVec>(out + 16, out_hi);
    }
}

bool aligned16(const void *pointer) { return (reinterpret_cast<uintptr_t>(pointer) & 15u) == 0; }
bool strides4(RocmKernelsStrides s) { return s.batch % 4 == 0 && s.head % 4 == 0 && s.token % 4 == 0; }

template <bool kBackward>
int launch(const RotaryArgs &a, bool vec, cudaStream_t stream) {
    const unsigned long long threads = 4ull * a.rows;
    const unsigned blocks = static_cast<unsigned>((threads + 255) / 256);
    if (vec)
        rotary_kernel<kBackward, true><<<blocks, 256, 0, stream>>>(a);
    else
        rotary_kernel<kBackward, false><<<blocks, 256, 0, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace

extern "C" int rotary_fp32(const float *q, const float *k, const float *cos, const float *sin, float *oq, float *ok, int batch,
                           int heads, int length, int backward, RocmKernelsStrides qs, RocmKernelsStrides ks,
                           RocmKernelsStrides cs, RocmKernelsStrides ss, RocmKernelsStream stream) {
    if (!q || !k || !cos || !sin || !oq || !ok || batch <= 0 || heads <= 0 || length <= 0) return cudaErrorInvalidValue;
    const long long rows = static_cast<long long>(batch) * heads * length;
    if (rows > INT_MAX / 4) return cudaErrorInvalidValue;  // thread index in 32 bits (2^29 rows = 64 GiB per tensor)
    RotaryArgs a{};
    a.q = q, a.k = k, a.cos = cos, a.sin = sin, a.oq = oq, a.ok = ok;
    a.qb = qs.batch, a.qh = qs.head, a.qt = qs.token;
    a.kb = ks.batch, a.kh = ks.head, a.kt = ks.token;
    a.cb = cs.batch, a.ct = cs.token, a.sb = ss.batch, a.st = ss.token;
    a.heads = heads, a.length = length;
    a.rows = static_cast<unsigned>(rows);
    const bool vec = aligned16(q) && aligned16(k) && aligned16(cos) && aligned16(sin) && aligned16(oq) && aligned16(ok) &&
                     strides4(qs) && strides4(ks) && cs.batch % 4 == 0 && cs.token % 4 == 0 && ss.batch % 4 == 0 &&
                     ss.token % 4 == 0;
    return backward ? launch<true>(a, vec, stream) : launch<false>(a, vec, stream);
}
