// Shared-memory layouts of the split-FP16 tensor-core operands (sm_100a), shared by the flash
// forward and the backward.
//
//   FP32 tiles as TMA lands them: 64 rows x D features as D / 32 boxes of 64 rows x 32 features
//   (128 bytes per row, 128B swizzle: 16-byte chunk c of row r at r * 8 + (c ^ (r % 8))).
//   Row layout (K-major B operand over the features): row r holds x0 (D FP16) and x1 (D FP16);
//   for D = 32 both halves share one 128-byte row ([x0 | x1]), for D = 64 x0 and x1 are separate
//   64 x 128-byte tiles. 128B swizzle. Read MN-major it is also the B operand over the 64 rows
//   (each row one K index, [x0 | x1] its 2D MN elements): the backward's X products.
//   Transposed layout (K-major B operand over the 64 rows, the forward's V): feature rows f (x0)
//   and D + f (x1), each 64 FP16 (128 bytes), rows 8g..8g+7 of the source tile in 16-byte chunk
//   g. 128B swizzle.
#pragma once

#include "tc_primitives.cuh"

namespace rk {
namespace tc {

constexpr int kBoxRows = 64;
constexpr int kBoxFloats = kBoxRows * 32;  // one TMA box: 64 rows x 32 FP32 (8 KB)
constexpr int kBoxBytes = kBoxFloats * 4;

// x' = (a, b) * scale split into FP16 pairs: p0 = FP16(x') rounded to nearest (11 significant
// bits), p1 = FP16(x' - p0), the residual taken from p0 widened back, so it is exact in FP32 before
// its own rounding. Low halves hold a. kPairs: the multiply and subtract as packed FP32 pairs (three
// issue slots per value instead of four; needs register pairs, which the d = 32 forward's split
// warps cannot spare without spilling).
template <bool kPairs>
__device__ __forceinline__ void split_pack2(float a, float b, float scale, uint32_t &p0, uint32_t &p1) {
    if constexpr (kPairs) {
        const float2 scaled = mul_f32x2(make_float2(a, b), make_float2(scale, scale));
        p0 = pack_half2(scaled.x, scaled.y);
        const float2 residual = sub_f32x2(scaled, unpack_half2(p0));
        p1 = pack_half2(residual.x, residual.y);
    } else {
        const float sa = a * scale, sb = b * scale;
        p0 = pack_half2(sa, sb);
        const float2 widened = unpack_half2(p0);
        p1 = pack_half2(sa - widened.x, sb - widened.y);
    }
}

// Eight values (scaled) as the 16-byte FP16 chunks of x0 and x1 (split_pack2 per pair).
template <bool kPairs>
__device__ __forceinline__ void split_pack8(const float (&x)[8], float scale, uint4 &x0, uint4 &x1) {
    split_pack2<kPairs>(x[0], x[1], scale, x0.x, x1.x);
    split_pack2<kPairs>(x[2], x[3], scale, x0.y, x1.y);
    split_pack2<kPairs>(x[4], x[5], scale, x0.z, x1.z);
    split_pack2<kPairs>(x[6], x[7], scale, x0.w, x1.w);
}

// 16-byte chunk `chunk` (features 4 chunk .. 4 chunk + 3) of row `row` of an FP32 tile.
template <int D>
__device__ __forceinline__ float4 raw_chunk(const float *tile, int row, int chunk) {
    const float4 *box = reinterpret_cast<const float4 *>(tile) + (chunk >> 3) * (kBoxFloats / 4);
    return box[row * 8 + ((chunk & 7) ^ (row & 7))];
}

// Row layout: the 16-byte FP16 chunk m (features 8m..8m+7) of part x0 (part 0) or x1 (part 1)
// of row `row`.
template <int D>
__device__ __forceinline__ uint4 *row_chunk(uint32_t *tile, int row, int part, int m) {
    if constexpr (D == 32)
        return reinterpret_cast<uint4 *>(tile) + row * 8 + ((4 * part + m) ^ (row & 7));
    else
        return reinterpret_cast<uint4 *>(tile) + part * (kBoxBytes / 16) + row * 8 + (m ^ (row & 7));
}

// Descriptor offset (16-byte units) of the x1 part of a row-layout tile.
template <int D>
constexpr uint64_t row_x1_offset() {
    return D == 32 ? 4 : kBoxBytes / 16;
}

// Key tiles (of 64 keys) of the window [first, last) up to its last visible key (mask[key] != 0), 0 when every
// key is masked: the warp reads the mask backwards from `last`, 128 keys (4 per lane) at a time.
// Warp-collective; every lane returns the count.
__device__ __forceinline__ int visible_tiles_of(const unsigned char *mask, int first, int last, int lane) {
    int end = last;
    while (end > first) {
        const int lo = max(first, end - 128);
        int top = -1;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int key = end - 1 - 4 * lane - e;
            if (key >= lo && mask[key] != 0) top = max(top, key);
        }
        top = __reduce_max_sync(0xffffffffu, top);
        if (top >= 0) {
            end = top + 1;
            break;
        }
        end = lo;
    }
    return end > first ? (end - first + kBoxRows - 1) / kBoxRows : 0;
}

}  // namespace tc
}  // namespace rk
