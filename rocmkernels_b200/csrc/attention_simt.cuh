// Exact-FP32 SIMT attention kernels for sm_100a (head width 32 or 64).
//
// These are the FP32-FMA variants: every product and sum is an FP32 FFMA, so they carry no
// tensor-core rounding. They serve the simple, tiled, statistics and backward entries and are
// the parity anchor for the tcgen05 path.
//
// Structure (one CTA = 256 threads = 16 x 16 thread grid):
//   forward   : a CTA owns BQ = 64 queries and streams 64-key tiles of K/V through shared
//               memory. Each thread computes a 4 x 4 block of scores (4 query rows ty*4+i, keys
//               tx + 16*jj), the 16 threads of a row reduce max/sum with shuffles inside one
//               half-warp, P goes through shared memory and each thread accumulates 4 rows x
//               D/16 features of O. Online softmax as in the reference's flash body
//               (AttentionFlash32.h:96-112), with exp evaluated as exp2 on the MUFU unit.
//   backward  : the reference's two-kernel split (Attention.hip:205-223): a query-major kernel
//               computes delta = sum(dO * O) and dQ; a key-major kernel recomputes P from the
//               saved {max, sum} (lse) and accumulates dK and dV. Both recompute S and dP.
#pragma once

#include "attention_common.cuh"
#include "rotary.cuh"

namespace rk {
namespace simt {

constexpr int kThreads = 256;
constexpr int kBlockQ = 64;
constexpr int kBlockK = 64;
constexpr int kPitchP = kBlockK + 4;

template <int D> struct Shape {
    static constexpr int pitch = D + 4;    // padded row pitch of a [rows][D] tile (keeps float4 alignment)
    static constexpr int features = D / 16; // O / dQ / dK / dV features per thread (D = 16 only in the forward)
    static constexpr int tile = 64 * pitch; // floats in one 64-row tile
};

// dst[r][c] = scale * src(row0 + r, c) for rows below `limit` whose flag is set, else 0; T is the
// storage type (FP32, or FP16 widened to FP32).
template <int D, int ROWS, class T>
__device__ __forceinline__ void load_rows(float *dst, const T *src, long long stride, int row0, int limit, float scale,
                                          bool vec4, const int *flags) {
    constexpr int pitch = Shape<D>::pitch;
    if (vec4) {
        constexpr int per_row = D / 4;
        for (int index = threadIdx.x; index < ROWS * per_row; index += kThreads) {
            const int r = index / per_row, c4 = index % per_row;
            const int row = row0 + r;
            float4 value = make_float4(0.f, 0.f, 0.f, 0.f);
            if (row < limit && (flags == nullptr || flags[r])) {
                value = load4(src + (long long)row * stride + 4 * c4);
                value.x *= scale; value.y *= scale; value.z *= scale; value.w *= scale;
            }
            *reinterpret_cast<float4 *>(dst + r * pitch + c4 * 4) = value;
        }
    } else {
        for (int index = threadIdx.x; index < ROWS * D; index += kThreads) {
            const int r = index / D, c = index % D;
            const int row = row0 + r;
            float value = 0.f;
            if (row < limit && (flags == nullptr || flags[r])) value = load1(src + (long long)row * stride + c) * scale;
            dst[r * pitch + c] = value;
        }
    }
}

// acc[i][jj] += A[ty*4 + i] . B[tx + 16*jj] over D features (A, B: [64][pitch] tiles).
template <int D>
__device__ __forceinline__ void tile_dot(float (&acc)[4][4], const float *A, const float *B, int ty, int tx) {
    constexpr int pitch = Shape<D>::pitch;
#pragma unroll 2
    for (int c = 0; c < D; c += 4) {
        float4 a[4], b[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) a[i] = *reinterpret_cast<const float4 *>(A + (ty * 4 + i) * pitch + c);
#pragma unroll
        for (int j = 0; j < 4; ++j) b[j] = *reinterpret_cast<const float4 *>(B + (tx + 16 * j) * pitch + c);
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                acc[i][j] = fmaf(a[i].x, b[j].x, acc[i][j]);
                acc[i][j] = fmaf(a[i].y, b[j].y, acc[i][j]);
                acc[i][j] = fmaf(a[i].z, b[j].z, acc[i][j]);
                acc[i][j] = fmaf(a[i].w, b[j].w, acc[i][j]);
            }
    }
}

// out[i][f] += sum_j W[ty*4 + i][j] * X[j][tx*F + f] over 64 rows j (W: [64][kPitchP], X: [64][pitch]).
template <int D>
__device__ __forceinline__ void tile_accumulate(float (&out)[4][Shape<D>::features], const float *W, const float *X,
                                                int ty, int tx) {
    constexpr int pitch = Shape<D>::pitch;
    constexpr int F = Shape<D>::features;
#pragma unroll 2
    for (int j = 0; j < kBlockK; j += 4) {
        float4 w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) w[i] = *reinterpret_cast<const float4 *>(W + (ty * 4 + i) * kPitchP + j);
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
            float x[F];
            if constexpr (F == 1) {
                x[0] = X[(j + jj) * pitch + tx];
            } else if constexpr (F == 2) {
                const float2 t = *reinterpret_cast<const float2 *>(X + (j + jj) * pitch + tx * 2);
                x[0] = t.x; x[1] = t.y;
            } else {
                const float4 t = *reinterpret_cast<const float4 *>(X + (j + jj) * pitch + tx * 4);
                x[0] = t.x; x[1] = t.y; x[2] = t.z; x[3] = t.w;
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float weight = jj == 0 ? w[i].x : jj == 1 ? w[i].y : jj == 2 ? w[i].z : w[i].w;
#pragma unroll
                for (int f = 0; f < F; ++f) out[i][f] = fmaf(weight, x[f], out[i][f]);
            }
        }
    }
}

// Rotary prologue on a staged [64][pitch] tile of 32-wide rows (rows row0.. of batch b; rows at
// or past `limit` are zero and stay zero): features f and f + 16 rotate by the tables of their
// token (rotate_pair, the rotary_fp32 forward), then everything is multiplied by `scale`.
template <int D>
__device__ __forceinline__ void rotate_tile(float *tile, int b, int row0, int limit, const AttentionParams &p, float scale) {
    static_assert(D == 32, "the rotary embedding is defined for 32-wide heads");
    constexpr int pitch = Shape<D>::pitch;
    for (int index = threadIdx.x; index < 64 * 16; index += kThreads) {
        const int r = index >> 4, f = index & 15;
        const int row = row0 + r;
        if (row >= limit) continue;
        const float *c = p.cos_row(b, row), *sn = p.sin_row(b, row);
        float lo, hi;
        rotate_pair<false>(tile[r * pitch + f], tile[r * pitch + f + 16], __ldg(c + f), __ldg(c + f + 16), __ldg(sn + f),
                           __ldg(sn + f + 16), lo, hi);
        tile[r * pitch + f] = lo * scale;
        tile[r * pitch + f + 16] = hi * scale;
    }
}

__device__ __forceinline__ float half_warp_max(float value) {
#pragma unroll
    for (int offset = 8; offset; offset >>= 1) value = fmaxf(value, __shfl_xor_sync(0xffffffffu, value, offset));
    return value;
}

__device__ __forceinline__ float half_warp_sum(float value) {
#pragma unroll
    for (int offset = 8; offset; offset >>= 1) value += __shfl_xor_sync(0xffffffffu, value, offset);
    return value;
}

__device__ __forceinline__ void decode_block(int block, int blocks_per_head, int heads, int &tile, int &h, int &b) {
    tile = block % blocks_per_head;
    const int bh = block / blocks_per_head;
    h = bh % heads;
    b = bh / heads;
}

// ------------------------------------------------------------------------------------------
// Forward: O = softmax(scale * Q K^T, masked) V and lse = {max, sum}; STATS_ONLY skips V and O.
// Replaces attention_query<false> (Attention.hip:32-115), attention_query_tiled<false>
// (AttentionTile32.h:12-217) and attention64_query<false> (Attention64.hip:34-129); with T =
// __half or D = 16 it is the exact-FP32 path of the generic forward (attention_generic_query and
// attention_generic_query_half, AttentionGeneric.hip:36-237): FP16 storage is widened on load,
// every product and sum is FP32, O is rounded to the storage type on the store. kRotary: q and
// k rows are rotated (rotary_fp32's forward, Rotary.hip:37-40) as they are staged.
// ------------------------------------------------------------------------------------------
template <int D, bool STATS_ONLY>
struct ForwardSmem {
    static constexpr int floats = Shape<D>::tile * (STATS_ONLY ? 2 : 3) + (STATS_ONLY ? 0 : kBlockQ * kPitchP) + kBlockK;
    static constexpr int bytes = floats * 4;
};

template <int D, bool STATS_ONLY, class T = float, bool kRotary = false>
__global__ void __launch_bounds__(kThreads) forward_kernel(AttentionParams p) {
    extern __shared__ float4 shared_raw[];
    float *Qs = reinterpret_cast<float *>(shared_raw);
    float *Ks = Qs + Shape<D>::tile;
    float *Vs = Ks + Shape<D>::tile;
    float *Ps = STATS_ONLY ? Vs : Vs + Shape<D>::tile;
    int *flags = reinterpret_cast<int *>(STATS_ONLY ? Vs : Ps + kBlockQ * kPitchP);
    constexpr int F = Shape<D>::features;

    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int blocks_per_head = (p.queries + kBlockQ - 1) / kBlockQ;
    int tile, h, b;
    decode_block(blockIdx.x, blocks_per_head, p.heads, tile, h, b);
    const int q0 = tile * kBlockQ;
    const unsigned char *mask = p.mask + (long long)b * p.keys;

    load_rows<D, kBlockQ>(Qs, p.q.row_as<T>(b, h, 0), p.q.st, q0, p.queries, kRotary ? 1.f : p.scale, p.vec4, nullptr);
    if constexpr (kRotary) {
        __syncthreads();
        rotate_tile<D>(Qs, b, q0, p.queries, p, p.scale);
    }

    float m[4], l[4], o[4][F];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        m[i] = -INFINITY;
        l[i] = 0.f;
#pragma unroll
        for (int f = 0; f < F; ++f) o[i][f] = 0.f;
    }

    int first, last;
    key_window(q0, q0 + kBlockQ, p.keys, p.radius, first, last);
    for (int k0 = first; k0 < last; k0 += kBlockK) {
        __syncthreads();  // previous tile consumed (and Q stored on the first pass)
        int visible = 0;
        if (threadIdx.x < kBlockK) {
            const int key = k0 + threadIdx.x;
            visible = key < last && mask[key] != 0;
            flags[threadIdx.x] = visible;
        }
        if (!__syncthreads_or(visible)) continue;  // whole tile masked: contributes nothing
        load_rows<D, kBlockK>(Ks, p.k.row_as<T>(b, h, 0), p.k.st, k0, last, 1.f, p.vec4, flags);
        if constexpr (!STATS_ONLY) load_rows<D, kBlockK>(Vs, p.v.row_as<T>(b, h, 0), p.v.st, k0, last, 1.f, p.vec4, flags);
        __syncthreads();
        if constexpr (kRotary) {
            rotate_tile<D>(Ks, b, k0, last, p, 1.f);
            __syncthreads();
        }

        float s[4][4] = {};
        tile_dot<D>(s, Qs, Ks, ty, tx);

#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int query = q0 + ty * 4 + i;
            float tile_max = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int column = tx + 16 * j;
                const bool active = flags[column] && query < p.queries && in_window(query, k0 + column, p.radius);
                if (!active) s[i][j] = -INFINITY;
                tile_max = fmaxf(tile_max, s[i][j]);
            }
            const float next = fmaxf(m[i], half_warp_max(tile_max));
            const float old_weight = isfinite(m[i]) ? fast_exp2((m[i] - next) * kLog2e) : 0.f;
            const float offset = -next * kLog2e;
            float row_sum = 0.f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                s[i][j] = s[i][j] == -INFINITY ? 0.f : fast_exp2(fmaf(s[i][j], kLog2e, offset));
                row_sum += s[i][j];
            }
            l[i] = l[i] * old_weight + half_warp_sum(row_sum);
            m[i] = next;
#pragma unroll
            for (int f = 0; f < F; ++f) o[i][f] *= old_weight;
        }
        if constexpr (!STATS_ONLY) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) Ps[(ty * 4 + i) * kPitchP + tx + 16 * j] = s[i][j];
            __syncwarp();  // the 16 threads of a row group live in one half-warp
            tile_accumulate<D>(o, Ps, Vs, ty, tx);
        }
    }

    // Epilogue (AttentionFlash32.h:157-169): O = acc / total; fully masked rows give O = 0 and
    // {-inf, 0}; a NaN total propagates, or gives 0 and {-inf, 0} when p.zero_nan_rows is set.
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int query = q0 + ty * 4 + i;
        if (query >= p.queries) continue;
        const float total = l[i];
        const bool nan_out = isnan(total) && !p.zero_nan_rows;
        if constexpr (!STATS_ONLY) {
            T *out = p.o.row_as<T>(b, h, query) + tx * F;
#pragma unroll
            for (int f = 0; f < F; ++f) store1(out + f, total > 0.f ? o[i][f] / total : nan_out ? NAN : 0.f);
        }
        if (tx == 0) {
            const long long row = ((long long)b * p.heads + h) * p.queries + query;
            p.lse[row * 2] = total > 0.f ? m[i] : nan_out ? NAN : -INFINITY;
            p.lse[row * 2 + 1] = total > 0.f ? total : nan_out ? NAN : 0.f;
        }
    }
}

// ------------------------------------------------------------------------------------------
// Backward, query-major pass. MODE selects what it produces:
//   kDeltaAndDq  : delta = sum_c dO*O per row (written), then dQ          (Attention.hip:32-115, BACKWARD)
//   kSoftmaxDelta: delta = sum_j P_ij * (dO_i . v_j) only, no O read      (AttentionTile32.h STATISTICS_ONLY)
//   kDqFromDelta : dQ with delta read from the buffer                     (AttentionTile32.h SOFTMAX_DELTA)
// P_ij = exp(s_ij - max_i) / sum_i from the saved lse; dS = P * (dP - delta); dQ = scale * dS K.
// ------------------------------------------------------------------------------------------
enum QueryMode { kDeltaAndDq = 0, kSoftmaxDelta = 1, kDqFromDelta = 2 };

template <int D>
struct QuerySmem {
    static constexpr int floats = Shape<D>::tile * 4 + kBlockQ * kPitchP + kBlockK + kBlockQ;
    static constexpr int bytes = floats * 4;
};

template <int D, int MODE>
__global__ void __launch_bounds__(kThreads, 1) backward_query_kernel(AttentionParams p) {
    extern __shared__ float4 shared_raw[];
    float *Qs = reinterpret_cast<float *>(shared_raw);
    float *dOs = Qs + Shape<D>::tile;
    float *Ks = dOs + Shape<D>::tile;
    float *Vs = Ks + Shape<D>::tile;
    float *dSs = Vs + Shape<D>::tile;
    int *flags = reinterpret_cast<int *>(dSs + kBlockQ * kPitchP);
    float *delta_s = reinterpret_cast<float *>(flags + kBlockK);
    constexpr int F = Shape<D>::features;
    constexpr int pitch = Shape<D>::pitch;

    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int blocks_per_head = (p.queries + kBlockQ - 1) / kBlockQ;
    int tile, h, b;
    decode_block(blockIdx.x, blocks_per_head, p.heads, tile, h, b);
    const int q0 = tile * kBlockQ;
    const long long row_base = ((long long)b * p.heads + h) * p.queries;
    const unsigned char *mask = p.mask + (long long)b * p.keys;

    load_rows<D, kBlockQ>(Qs, p.q.row(b, h, 0), p.q.st, q0, p.queries, p.scale, p.vec4, nullptr);
    load_rows<D, kBlockQ>(dOs, p.dout.row(b, h, 0), p.dout.st, q0, p.queries, 1.f, p.vec4, nullptr);
    if constexpr (MODE == kDeltaAndDq) {
        // O staged in the K buffer, then delta per row (8 rows per warp).
        load_rows<D, kBlockQ>(Ks, p.o_in.row(b, h, 0), p.o_in.st, q0, p.queries, 1.f, p.vec4, nullptr);
        __syncthreads();
        for (int r = warp * 8; r < warp * 8 + 8; ++r) {
            float partial = 0.f;
#pragma unroll
            for (int c = lane; c < D; c += 32) partial = fmaf(dOs[r * pitch + c], Ks[r * pitch + c], partial);
#pragma unroll
            for (int offset = 16; offset; offset >>= 1) partial += __shfl_xor_sync(0xffffffffu, partial, offset);
            if (lane == 0) {
                delta_s[r] = partial;
                if (q0 + r < p.queries) p.delta[row_base + q0 + r] = partial;
            }
        }
    } else if constexpr (MODE == kDqFromDelta) {
        if (threadIdx.x < kBlockQ) {
            const int query = q0 + threadIdx.x;
            delta_s[threadIdx.x] = query < p.queries ? p.delta[row_base + query] : 0.f;
        }
    }
    __syncthreads();

    float row_max[4], inv_total[4], row_delta[4], acc[4][F], softmax_delta[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int query = q0 + ty * 4 + i;
        const bool valid = query < p.queries;
        row_max[i] = valid ? p.lse_in[(row_base + query) * 2] : -INFINITY;
        inv_total[i] = valid ? 1.f / p.lse_in[(row_base + query) * 2 + 1] : 0.f;
        row_delta[i] = MODE == kSoftmaxDelta ? 0.f : delta_s[ty * 4 + i];
        softmax_delta[i] = 0.f;
#pragma unroll
        for (int f = 0; f < F; ++f) acc[i][f] = 0.f;
    }

    int first, last;
    key_window(q0, q0 + kBlockQ, p.keys, p.radius, first, last);
    for (int k0 = first; k0 < last; k0 += kBlockK) {
        __syncthreads();
        int visible = 0;
        if (threadIdx.x < kBlockK) {
            const int key = k0 + threadIdx.x;
            visible = key < last && mask[key] != 0;
            flags[threadIdx.x] = visible;
        }
        if (!__syncthreads_or(visible)) continue;
        load_rows<D, kBlockK>(Ks, p.k.row(b, h, 0), p.k.st, k0, last, 1.f, p.vec4, flags);
        load_rows<D, kBlockK>(Vs, p.v.row(b, h, 0), p.v.st, k0, last, 1.f, p.vec4, flags);
        __syncthreads();

        float s[4][4] = {}, dp[4][4] = {};
        tile_dot<D>(s, Qs, Ks, ty, tx);
        tile_dot<D>(dp, dOs, Vs, ty, tx);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int query = q0 + ty * 4 + i;
            const float offset = -row_max[i] * kLog2e;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int column = tx + 16 * j;
                const bool active = flags[column] && query < p.queries && in_window(query, k0 + column, p.radius) &&
                                    row_max[i] != -INFINITY;
                const float probability = active ? fast_exp2(fmaf(s[i][j], kLog2e, offset)) * inv_total[i] : 0.f;
                if constexpr (MODE == kSoftmaxDelta) softmax_delta[i] = fmaf(probability, dp[i][j], softmax_delta[i]);
                else s[i][j] = probability * (dp[i][j] - row_delta[i]);
            }
        }
        if constexpr (MODE != kSoftmaxDelta) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) dSs[(ty * 4 + i) * kPitchP + tx + 16 * j] = s[i][j];
            __syncwarp();
            tile_accumulate<D>(acc, dSs, Ks, ty, tx);
        }
    }

#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int query = q0 + ty * 4 + i;
        if constexpr (MODE == kSoftmaxDelta) {
            const float total = half_warp_sum(softmax_delta[i]);
            if (tx == 0 && query < p.queries) p.delta[row_base + query] = total;
        } else {
            if (query >= p.queries) continue;
            float *out = p.dq + (row_base + query) * D + tx * F;
#pragma unroll
            for (int f = 0; f < F; ++f) out[f] = acc[i][f] * p.scale;
        }
    }
}

// ------------------------------------------------------------------------------------------
// Backward, key-major pass: dV = P^T dO, dK = scale * dS^T Q, recomputing P from lse and reading
// delta. Replaces attention_key_value (Attention.hip:117-169), attention_single_query_kv
// (:171-189), attention_key_value_tiled (AttentionTile32.h:219-311) and attention64_key_value
// (Attention64.hip:131-191). Masked keys are loaded as zero rows, so their dK and dV are 0.
// ------------------------------------------------------------------------------------------
template <int D>
struct KeySmem {
    static constexpr int floats = Shape<D>::tile * 4 + 2 * kBlockK * kPitchP + 3 * kBlockQ + kBlockK;
    static constexpr int bytes = floats * 4;
};

template <int D>
__global__ void __launch_bounds__(kThreads, 1) backward_key_kernel(AttentionParams p) {
    extern __shared__ float4 shared_raw[];
    float *Ks = reinterpret_cast<float *>(shared_raw);
    float *Vs = Ks + Shape<D>::tile;
    float *Qs = Vs + Shape<D>::tile;
    float *dOs = Qs + Shape<D>::tile;
    float *Ps = dOs + Shape<D>::tile;
    float *dSs = Ps + kBlockK * kPitchP;
    float *max_s = dSs + kBlockK * kPitchP;
    float *inv_s = max_s + kBlockQ;
    float *delta_s = inv_s + kBlockQ;
    int *flags = reinterpret_cast<int *>(delta_s + kBlockQ);
    constexpr int F = Shape<D>::features;

    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int blocks_per_head = (p.keys + kBlockK - 1) / kBlockK;
    int tile, h, b;
    decode_block(blockIdx.x, blocks_per_head, p.heads, tile, h, b);
    const int k0 = tile * kBlockK;
    const long long row_base = ((long long)b * p.heads + h) * p.queries;
    const long long key_base = ((long long)b * p.heads + h) * p.keys;
    const unsigned char *mask = p.mask + (long long)b * p.keys;

    int visible = 0;
    if (threadIdx.x < kBlockK) {
        const int key = k0 + threadIdx.x;
        visible = key < p.keys && mask[key] != 0;
        flags[threadIdx.x] = visible;
    }
    const bool any_visible = __syncthreads_or(visible);

    float acc_k[4][F], acc_v[4][F];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int f = 0; f < F; ++f) acc_k[i][f] = acc_v[i][f] = 0.f;

    if (any_visible) {
        load_rows<D, kBlockK>(Ks, p.k.row(b, h, 0), p.k.st, k0, p.keys, 1.f, p.vec4, flags);
        load_rows<D, kBlockK>(Vs, p.v.row(b, h, 0), p.v.st, k0, p.keys, 1.f, p.vec4, flags);
        int first, last;  // queries that can see this key block
        key_window(k0, k0 + kBlockK, p.queries, p.radius, first, last);
        for (int i0 = first; i0 < last; i0 += kBlockQ) {
            __syncthreads();
            load_rows<D, kBlockQ>(Qs, p.q.row(b, h, 0), p.q.st, i0, last, p.scale, p.vec4, nullptr);
            load_rows<D, kBlockQ>(dOs, p.dout.row(b, h, 0), p.dout.st, i0, last, 1.f, p.vec4, nullptr);
            if (threadIdx.x < kBlockQ) {
                const int query = i0 + threadIdx.x;
                const bool valid = query < last;
                max_s[threadIdx.x] = valid ? p.lse_in[(row_base + query) * 2] : -INFINITY;
                inv_s[threadIdx.x] = valid ? 1.f / p.lse_in[(row_base + query) * 2 + 1] : 0.f;
                delta_s[threadIdx.x] = valid ? p.delta[row_base + query] : 0.f;
            }
            __syncthreads();

            float s[4][4] = {}, dp[4][4] = {};
            tile_dot<D>(s, Ks, Qs, ty, tx);   // s[i][jj] = k_(ty*4+i) . q_(tx+16jj) * scale
            tile_dot<D>(dp, Vs, dOs, ty, tx); // dp[i][jj] = v . dO
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int column = tx + 16 * j;
                const int query = i0 + column;
                const float maximum = max_s[column];
                const float offset = -maximum * kLog2e;
                const float inv = inv_s[column];
                const float dl = delta_s[column];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int key = k0 + ty * 4 + i;
                    const bool active = flags[ty * 4 + i] && query < last && in_window(query, key, p.radius) &&
                                        maximum != -INFINITY;
                    const float probability = active ? fast_exp2(fmaf(s[i][j], kLog2e, offset)) * inv : 0.f;
                    s[i][j] = probability;
                    dp[i][j] = probability * (dp[i][j] - dl);
                }
            }
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    Ps[(ty * 4 + i) * kPitchP + tx + 16 * j] = s[i][j];
                    dSs[(ty * 4 + i) * kPitchP + tx + 16 * j] = dp[i][j];
                }
            __syncwarp();
            tile_accumulate<D>(acc_v, Ps, dOs, ty, tx);
            tile_accumulate<D>(acc_k, dSs, Qs, ty, tx);
        }
    }

#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int key = k0 + ty * 4 + i;
        if (key >= p.keys) continue;
        float *out_k = p.dk + (key_base + key) * D + tx * F;
        float *out_v = p.dv + (key_base + key) * D + tx * F;
#pragma unroll
        for (int f = 0; f < F; ++f) {
            out_k[f] = acc_k[i][f];
            out_v[f] = acc_v[i][f];
        }
    }
}

}  // namespace simt
}  // namespace rk
