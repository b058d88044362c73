// Tensor-core backward for head width 32 on sm_100a: tcgen05.mma (kind::f16) on split FP16
// operands with TMEM accumulators, TMA-staged tiles.
//
// Replaces the reference's backward pair (attention_query<true> for delta and dQ,
// Attention.hip:32-115, and attention_key_value, :117-169) with the same two-pass structure and
// results: P_ij = exp(s_ij - max_i) / sum_i from the saved lse, dS = P (dP - delta),
// dQ = scale dS K, dK = dS^T (scale Q), dV = P^T dO, delta_i = sum_c dO_ic O_ic; masked keys get
// dK = dV = 0.
//
// One kernel template, two roles. A CTA owns 128 "rows" (TMEM lanes) and walks 64-wide "column"
// tiles:
//   query rows (pass 1): rows = queries, columns = key tiles.   S = Q K^T, dP = dO V^T,
//                        X1 += dS K (dQ). Also writes delta.
//   key rows   (pass 2): rows = keys, columns = query tiles.    S^T = K Q^T, dP^T = V dO^T,
//                        X1 += dS^T Q (dK), X2 += P^T dO (dV).
// Warps: 0-3 row warps (thread = row = TMEM lane), 4 TMA producer, 5 MMA issuer (whole warp,
// elected issue), 6-7 split warps (FP16 conversion of each column tile). d = 32: two CTAs per
// SM (256 TMEM columns each); d = 64: one (512).
//
// Split FP16 operands as in the forward: every operand is scaled by a power of two so that its
// largest magnitude lies in [2^14, 2^15) (row operands per row, column tiles per tile, P by
// 2^14, dS per row and tile from the bound |dS| <= ||dO_i||_1 max|v| + |delta_i| (pass 1) or
// ||v_j||_1 max|dO| + max|delta| (pass 2), which needs no extra pass over dS) and split into
// x0 + x1: S = a0.b1 + a1.b0 + a0.b0 (6 MMAs N64 for d = 32). The X products read the column
// tile's row layout [b0 | b1] as an MN-major B operand: one MMA of N = 2D per 16 columns and
// term gives ds.b0 and ds.b1 side by side, X = (ds0 + ds1).[b0 | b1] (8 MMAs), and the fold adds
// the two halves -- no transposed copy of any tile. The per-tile products are folded into FP32
// registers (the tensor core's accumulation is not round-to-nearest), so the sums over column
// tiles are plain FP32.
//
// TMEM per row (d = 32; d = 64 doubles every width but the 64-column S and dP):
//   query rows: a1 [x0 16 | x1 16] 0-31 | a2 32-63 | S 64-127 | dP then dS 128-191 | X1 [b0 | b1] 192-255
//   key rows:   S then P 0-63 | dP then dS 64-127 | X1 [b0 | b1] 128-191 | X2 192-255, the row
//               operands (K, V) in shared memory as the K-major A of S^T and dP^T (the d = 64
//               key-rows pass keeps them in TMEM, 512 columns)
// P and dS overwrite S and dP chunk by chunk: 16 columns [x0 pairs 8 | x1 pairs 8], which
// occupy exactly the 16 columns of scores the chunk has just read.
#include "attention_tc.cuh"

#include <cudaTypedefs.h>

#include <mutex>

#include "tc_operands.cuh"

namespace rk {
namespace tc {

namespace {

// Optional pipeline timeline (build with -DRK_TC_TRACE; compiled out otherwise): clock64 stamps
// of CTA 0 of each pass per column tile and role, read back with rocmkernels_attention_backward_trace().
#ifdef RK_TC_TRACE
constexpr int kTraceTiles = 64, kTraceEvents = 16;
__device__ long long g_bwd_trace[2][kTraceTiles][kTraceEvents];
#define RK_BTRACE(tile_index, event)                                                                              \
    do {                                                                                                         \
        if (blockIdx.x == 0 && (tile_index) < kTraceTiles) g_bwd_trace[kKeyRows][(tile_index)][(event)] = clock64(); \
    } while (0)
#define RK_FTRACE(tile_index, event)                                                                    \
    do {                                                                                               \
        if (blockIdx.x == 0 && (tile_index) < kTraceTiles) g_bwd_trace[0][(tile_index)][(event)] = clock64(); \
    } while (0)
#else
#define RK_BTRACE(tile_index, event) \
    do {                            \
    } while (0)
#define RK_FTRACE(tile_index, event) \
    do {                            \
    } while (0)
#endif

constexpr int kRows = 128;
constexpr int kCols = 64;
constexpr int kThreads = 256;
constexpr int kProducerWarp = 4;
constexpr int kMmaWarp = 5;
constexpr int kSplitWarp = 6;
constexpr int kSplitThreads = 64;
constexpr uint32_t kIdescS = f16_instr_desc(128, 64);
constexpr uint64_t kDescStep = 2;  // one K=16 step of FP16 = 32 bytes

// Layout constants for head width D (32 or 64).
template <int D>
struct Geometry {
    static constexpr int kBoxes = D / 32;                   // TMA boxes per tile row
    static constexpr int kRawFloats = kBoxes * kBoxFloats;   // FP32 tile: kBoxes boxes of 64 x 32
    static constexpr int kRowWords = 64 * D;                // row layout: 64 rows x [x0 | x1] (2 D fp16 each)
    // Row layout: D = 32 keeps [x0 | x1] in one 128-byte row; D = 64 uses an x0 tile and an x1
    // tile of 64 rows x 128 bytes each. Descriptor offset (16-byte units) of the x1 part.
    static constexpr uint64_t kDescX1 = row_x1_offset<D>();
    static constexpr uint32_t kTmemColumns = D == 32 ? 256 : 512;
    static constexpr int kCtasPerSm = D == 32 ? 2 : 1;
    // X = dS.[b0 | b1]: B = the column tile's row layout read MN-major (N = 2D); for D = 64 the
    // x1 part (MN elements 64..127) is the next 8 KB tile.
    static constexpr uint32_t kIdescX = f16_instr_desc_b_mn(128, 2 * D);
    static constexpr uint32_t kMnChunkBytes = D == 32 ? 1024 : kBoxBytes;
};

// TMEM columns per row. The d = 32 key-rows pass keeps its row operands (K, V) in shared memory:
// its 256 columns hold S, dP and the two 2D-wide X products.
template <int D, bool kKeyRows>
struct Columns {
    static constexpr bool kRowOperandsInSmem = kKeyRows && D == 32;
    static constexpr uint32_t kA1 = 0, kA2 = D;
    static constexpr uint32_t kS = kRowOperandsInSmem ? 0 : 2 * D, kDP = kS + 64, kX1 = kS + 128, kX2 = kX1 + 2 * D;
    static_assert((kKeyRows ? kX2 : kX1) + 2 * D <= Geometry<D>::kTmemColumns, "TMEM budget");
    static_assert(kRowOperandsInSmem || (kA1 + D <= kA2 && kA2 + D <= kS), "row operands below S");
};

// Split FP16 row operands in shared memory (the d = 32 key-rows pass): K and V rows as
// 128 x [x0 | x1] (128 bytes per row), 128B swizzle -- the K-major A of S^T and dP^T.
template <int D, bool kInSmem>
struct alignas(1024) RowOperandTiles {
    uint32_t a1[kRows * D];  // K
    uint32_t a2[kRows * D];  // V
};
template <int D>
struct RowOperandTiles<D, false> {};

template <int D, bool kKeyRows>
struct alignas(1024) Storage {
    using G = Geometry<D>;
    // Pipeline depth: the key-rows pass spends the room of a third stage on its row operands.
    static constexpr int kStages = kKeyRows ? 2 : 3;
    float raw1[kStages][G::kRawFloats];                    // TMA tile: K (query rows) or Q (key rows), 128B swizzle
    float raw2[kStages][G::kRawFloats];                    // V or dO
    uint32_t b1[kStages][G::kRowWords];                    // raw1 rows as split FP16 (B of S; MN-major B of X1), 128B swizzle
    uint32_t b2[kStages][G::kRowWords];                    // raw2 rows (B of dP; key rows: MN-major B of X2)
    RowOperandTiles<D, Columns<D, kKeyRows>::kRowOperandsInSmem> a;  // d = 32 key rows: K, V
    alignas(16) float col_offset[kStages][kCols];          // key rows: 14 - max log2e - log2(sum) per query
    alignas(16) float col_delta[kStages][kCols];           // key rows: delta per query
    uint32_t col_mask[kStages][2];                         // visible columns
    int e1[kStages], e2[kStages];                          // tile scale exponents of raw1 (Q: of scale*Q) and raw2
    float col_delta_max[kStages];                          // key rows: max |delta| of the tile
    float split_max[2][2][3];                              // [tile parity][split warp]: max|raw1|, max|raw2|, max|delta|
    int split_ok[2][2];                                    // [tile parity][split warp]: its TMA wait succeeded
    uint64_t full[kStages];                                // TMA bytes landed
    uint64_t raw_free[kStages];                            // raw tiles converted: TMA may refill (64 arrivals)
    uint64_t ready[kStages];                               // conversion done (64 arrivals)
    uint64_t empty[kStages];                               // MMAs reading the stage finished (commit)
    uint64_t s_full;                                       // S and dP in TMEM (commit)
    uint64_t p_full;                                       // P / dS stored and the previous X folded (128 arrivals)
    uint64_t x_done;                                       // X1 (X2) of the tile in TMEM (commit)
    uint64_t rows_ready;                                   // row operands stored (128 arrivals)
    uint64_t mma_done;                                     // every MMA finished (commit)
    uint64_t range_ready;                                  // tile_count written (1 arrival)
    uint32_t tmem_base;
    int tile_count;                                        // column tiles visited
};

struct BackwardArgs {
    AttentionParams p;
    int blocks_per_head;  // row tiles per (batch, head)
};

__device__ __forceinline__ uint32_t lane_address(uint32_t base, int warp) {
    return base + (static_cast<uint32_t>((warp & 3) * 32) << 16);
}

// Splits a D-feature row (scaled by 2^exponent) and stores it to TMEM at `column` as FP16 pairs:
// x0 pairs in columns [0, D/2), x1 pairs in [D/2, D).
template <int D>
__device__ __forceinline__ void store_row_operand(const float (&x)[D], int exponent, uint32_t column) {
    const float scale = exp2_int(exponent);
#pragma unroll
    for (int half = 0; half < D / 32; ++half) {
        float a[16], b[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) {
            uint32_t p0, p1;
            split_pack2<false>(x[32 * half + 2 * c], x[32 * half + 2 * c + 1], scale, p0, p1);
            a[c] = __uint_as_float(p0);
            b[c] = __uint_as_float(p1);
        }
        tmem_store16x2(column + 16 * half, a, column + D / 2 + 16 * half, b);
    }
}

// The same into a shared-memory row layout (row `row` of a 128-row tile, 128B swizzle).
template <int D>
__device__ __forceinline__ void store_row_operand_smem(const float (&x)[D], int exponent, uint32_t *tile, int row) {
    const float scale = exp2_int(exponent);
#pragma unroll
    for (int m = 0; m < D / 8; ++m) {
        const float chunk[8] = {x[8 * m], x[8 * m + 1], x[8 * m + 2], x[8 * m + 3],
                                x[8 * m + 4], x[8 * m + 5], x[8 * m + 6], x[8 * m + 7]};
        uint4 c0, c1;
        split_pack8<false>(chunk, scale, c0, c1);
        *row_chunk<D>(tile, row, 0, m) = c0;
        *row_chunk<D>(tile, row, 1, m) = c1;
    }
}

// Loads a D-float row (zeros when !valid), multiplied by `scale`.
template <int D>
__device__ __forceinline__ void load_row(const float *row, bool valid, float scale, float (&x)[D]) {
    const float4 *r4 = reinterpret_cast<const float4 *>(row);
#pragma unroll
    for (int c = 0; c < D / 4; ++c) {
        const float4 v = valid ? __ldg(r4 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
        x[4 * c] = v.x * scale;
        x[4 * c + 1] = v.y * scale;
        x[4 * c + 2] = v.z * scale;
        x[4 * c + 3] = v.w * scale;
    }
}

template <int D>
__device__ __forceinline__ float abs_max(const float (&x)[D]) {
    float m = 0.f;
#pragma unroll
    for (int c = 0; c < D; c += 2) m = max3(m, fabsf(x[c]), fabsf(x[c + 1]));
    return m;
}

// S (N = 64) = a0.b1 + a1.b0 + a0.b0 over the D features; a at TMEM `a` ([x0 D/2 | x1 D/2]),
// b = the row layout (x0 part at b, x1 part at b + kDescX1). Commits to `bar` when given.
// Warp-collective.
template <int D>
__device__ __forceinline__ void issue_product(uint32_t d, uint32_t a, uint64_t b, uint64_t *bar) {
    constexpr uint64_t x1 = Geometry<D>::kDescX1;
    constexpr uint32_t h = D / 2;
    if constexpr (D == 32) {
        const uint32_t ga[4] = {a, a + 8, a + h, a + h + 8};
        const uint64_t gb[4] = {b + x1, b + x1 + kDescStep, b, b + kDescStep};
        mma4_f16_ts_warp(d, ga, gb, kIdescS, 1);
        if (bar != nullptr)
            mma2_f16_ts_commit_warp(d, a, a + 8, b, b + kDescStep, kIdescS, bar);
        else
            mma2_f16_ts_warp(d, a, a + 8, b, b + kDescStep, kIdescS);
    } else {
        const uint32_t g1a[4] = {a, a + 8, a + 16, a + 24};  // a0 . b1
        const uint64_t g1b[4] = {b + x1, b + x1 + kDescStep, b + x1 + 2 * kDescStep, b + x1 + 3 * kDescStep};
        mma4_f16_ts_warp(d, g1a, g1b, kIdescS, 1);
        const uint32_t g2a[4] = {a + h, a + h + 8, a + h + 16, a + h + 24};  // a1 . b0
        const uint64_t g2b[4] = {b, b + kDescStep, b + 2 * kDescStep, b + 3 * kDescStep};
        mma4_f16_ts_warp(d, g2a, g2b, kIdescS, 0);
        const uint32_t g3a[4] = {a, a + 8, a + 16, a + 24};  // a0 . b0
        if (bar != nullptr)
            mma4_f16_ts_commit_warp(d, g3a, g2b, kIdescS, 0, bar);
        else
            mma4_f16_ts_warp(d, g3a, g2b, kIdescS, 0);
    }
}

// The same with the row operand in shared memory (D = 32): `a` = descriptor of its row layout
// ([x0 | x1] per 128-byte row, x1 at +64 bytes).
template <int D>
__device__ __forceinline__ void issue_product_smem(uint32_t d, uint64_t a, uint64_t b, uint64_t *bar) {
    static_assert(D == 32, "shared-memory row operands: d = 32 only");
    constexpr uint64_t x1 = Geometry<D>::kDescX1;
    const uint64_t ga[4] = {a, a + kDescStep, a + x1, a + x1 + kDescStep};  // a0 . b1, a1 . b0
    const uint64_t gb[4] = {b + x1, b + x1 + kDescStep, b, b + kDescStep};
    mma4_f16_ss_warp(d, ga, gb, kIdescS, 1);
    const uint64_t ha[2] = {a, a + kDescStep};  // a0 . b0
    const uint64_t hb[2] = {b, b + kDescStep};
    if (bar != nullptr)
        mma2_f16_ss_commit_warp(d, ha, hb, kIdescS, bar);
    else
        mma2_f16_ss_warp(d, ha, hb, kIdescS);
}

// Splits 16 values (columns of a chunk) into FP16 pairs and stores them, without waiting, as
// [x0 pairs 8 | x1 pairs 8] at TMEM `chunk` (the A layout of one K=16 step).
__device__ __forceinline__ void store_split_chunk(uint32_t chunk, const float (&v)[16]) {
    float q0[8], q1[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        const float x0 = __uint_as_float(__float_as_uint(v[2 * c]) & 0xFFFFE000u);
        const float y0 = __uint_as_float(__float_as_uint(v[2 * c + 1]) & 0xFFFFE000u);
        const float2 residual = sub_f32x2(make_float2(v[2 * c], v[2 * c + 1]), make_float2(x0, y0));
        q0[c] = __uint_as_float(pack_half2(x0, y0));
        q1[c] = __uint_as_float(pack_half2(residual.x, residual.y));
    }
    tmem_store8x2_async(chunk, q0, chunk + 8, q1);
}

// X (N = 2D) = (x0 + x1).[b0 | b1] over the 64 columns: A chunks of 16 columns at
// `chunks` + 16 kk ([x0 pairs 8 | x1 pairs 8]), B = the column tile's row layout read MN-major
// (for each column a row of [b0 | b1]; 16 columns = 2048 bytes), so the products with b0 land
// in accumulator columns 0..D-1 and those with b1 in D..2D-1. Commits to `bar` when given.
// Warp-collective.
template <int D>
__device__ __forceinline__ void issue_x(uint32_t d, uint32_t chunks, uint64_t b, uint64_t *bar) {
    constexpr uint32_t idesc = Geometry<D>::kIdescX;
    constexpr uint64_t step = 2048 / 16;
    const uint32_t g1a[4] = {chunks, chunks + 8, chunks + 16, chunks + 24};
    const uint64_t g1b[4] = {b, b, b + step, b + step};
    mma4_f16_ts_warp(d, g1a, g1b, idesc, 1);
    const uint32_t g2a[4] = {chunks + 32, chunks + 40, chunks + 48, chunks + 56};
    const uint64_t g2b[4] = {b + 2 * step, b + 2 * step, b + 3 * step, b + 3 * step};
    if (bar != nullptr)
        mma4_f16_ts_commit_warp(d, g2a, g2b, idesc, 0, bar);
    else
        mma4_f16_ts_warp(d, g2a, g2b, idesc, 0);
}

// acc1 += X1 * scale1 (and acc2 += X2 * scale2 for key rows), eight columns at a time; each X
// holds the b0 and b1 products in columns 0..D-1 and D..2D-1.
template <int D, bool kKeyRows>
__device__ __forceinline__ void fold_x(float (&acc1)[D], float (&acc2)[kKeyRows ? D : 1], uint32_t lanes, float scale1,
                                       float scale2) {
    using C = Columns<D, kKeyRows>;
#pragma unroll
    for (int quarter = 0; quarter < D / 8; ++quarter) {
        float xa[8], xb[8];
        const float2 s1 = make_float2(scale1, scale1), s2 = make_float2(scale2, scale2);
        tmem_load8x2(lanes + C::kX1 + 8 * quarter, xa, lanes + C::kX1 + D + 8 * quarter, xb);
#pragma unroll
        for (int c = 0; c < 8; c += 2) {
            float *a = &acc1[8 * quarter + c];
            const float2 r = fma_f32x2(add_f32x2(make_float2(xa[c], xa[c + 1]), make_float2(xb[c], xb[c + 1])), s1, make_float2(a[0], a[1]));
            a[0] = r.x;
            a[1] = r.y;
        }
        if constexpr (kKeyRows) {
            tmem_load8x2(lanes + C::kX2 + 8 * quarter, xa, lanes + C::kX2 + D + 8 * quarter, xb);
#pragma unroll
            for (int c = 0; c < 8; c += 2) {
                float *a = &acc2[8 * quarter + c];
                const float2 r = fma_f32x2(add_f32x2(make_float2(xa[c], xa[c + 1]), make_float2(xb[c], xb[c + 1])), s2, make_float2(a[0], a[1]));
                a[0] = r.x;
                a[1] = r.y;
            }
        }
    }
}

// Converts the two FP32 tiles of one stage (split warps, 64 threads, row = 32 w + lane) to their
// row layouts: the B of S and dP, and read MN-major the B of X1 (and X2 for key rows); masked
// key rows zeroed (query rows).
template <int D, class St>
__device__ __forceinline__ void convert_stage(St &s, int stage, int w, int lane, bool keep_row, float scale_1, float scale_2) {
    const int row = 32 * w + lane;
#pragma unroll
    for (int which = 0; which < 2; ++which) {
        const float *raw = which == 0 ? s.raw1[stage] : s.raw2[stage];
        uint32_t *dst = which == 0 ? s.b1[stage] : s.b2[stage];
        const float scale = which == 0 ? scale_1 : scale_2;
#pragma unroll
        for (int m = 0; m < D / 8; ++m) {
            float4 lo = raw_chunk<D>(raw, row, 2 * m), hi = raw_chunk<D>(raw, row, 2 * m + 1);
            if (!keep_row) lo = hi = make_float4(0.f, 0.f, 0.f, 0.f);
            const float x[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
            uint4 c0, c1;
            split_pack8<true>(x, scale, c0, c1);
            *row_chunk<D>(dst, row, 0, m) = c0;
            *row_chunk<D>(dst, row, 1, m) = c1;
        }
    }
}

// The column tiles a CTA walks: its row tile [r0, r0 + 128) of row_count rows, the window
// [first, last) of columns that can see (or be seen by) it, window_tiles = 64-column tiles of the
// window, prefetched = those loaded before the mask is read.
struct TileWindow {
    int r0, row_count, first, last, window_tiles, prefetched, h, b;
    long long query_base;
    const unsigned char *mask;
};

// The CTA's row tile (blockIdx.x enumerates (batch, head, row tile), row tiles fastest) and its
// column window.
template <int kStages>
__device__ __forceinline__ TileWindow tile_window(const AttentionParams &p, bool key_rows, int blocks_per_head) {
    TileWindow t;
    int block = blockIdx.x;
    const int row_tile = block % blocks_per_head;
    block /= blocks_per_head;
    t.h = block % p.heads;
    t.b = block / p.heads;
    t.r0 = row_tile * kRows;
    t.row_count = key_rows ? p.keys : p.queries;
    const int column_count = key_rows ? p.queries : p.keys;
    key_window(t.r0, min(t.r0 + kRows, t.row_count), column_count, p.radius, t.first, t.last);
    t.window_tiles = t.last > t.first ? (t.last - t.first + kCols - 1) / kCols : 0;
    t.prefetched = min(t.window_tiles, kStages);
    t.query_base = (static_cast<long long>(t.b) * p.heads + t.h) * p.queries;
    t.mask = p.mask + static_cast<long long>(t.b) * p.keys;
    return t;
}

// Column tiles actually visited (published by the producer warp after its first loads).
// Query rows: the key window up to its last visible key (trailing key padding is skipped).
// Key rows: none when every key of the tile is masked (dK = dV = 0); else the query window.
template <class St>
__device__ __forceinline__ int visited_tiles(St &s) {
    return mbar_wait(&s.range_ready, 0) ? s.tile_count : 0;
}

// TMA producer warp (lane 0 issues): the raw FP32 column tiles into the stage ring, the visited
// tile count published on range_ready.
template <int D, bool kKeyRows, class St>
__device__ __forceinline__ void producer_role(St &s, const TileWindow &t, const CUtensorMap &tmap1, const CUtensorMap &tmap2,
                                              int lane) {
    using G = Geometry<D>;
    constexpr int kStages = St::kStages;
    const int first = t.first, last = t.last, window_tiles = t.window_tiles, prefetched = t.prefetched;
    const int r0 = t.r0, row_count = t.row_count, h = t.h, b = t.b;
    const unsigned char *mask = t.mask;
    const auto issue = [&](int j) {
        const int stage = j % kStages;
        RK_BTRACE(j, 0);
        mbar_arrive_expect_tx(&s.full[stage], 2 * G::kBoxes * kBoxBytes);
#pragma unroll
        for (int box = 0; box < G::kBoxes; ++box) {
            tma_load_4d(s.raw1[stage] + box * kBoxFloats, &tmap1, &s.full[stage], 32 * box, first + j * kCols, h, b);
            tma_load_4d(s.raw2[stage] + box * kBoxFloats, &tmap2, &s.full[stage], 32 * box, first + j * kCols, h, b);
        }
    };
    // The first stages go out before the mask is read.
    if (lane == 0)
        for (int j = 0; j < prefetched; ++j) issue(j);
    int tiles = window_tiles;
    if constexpr (kKeyRows) {
        bool visible = false;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int key = r0 + 4 * lane + e;
            visible = visible || (key < row_count && mask[key] != 0);
        }
        if (!__any_sync(0xffffffffu, visible)) tiles = 0;
    } else {
        tiles = visible_tiles_of(mask, first, last, lane);
    }
    if (lane == 0) {
        s.tile_count = tiles;
        mbar_arrive(&s.range_ready);
        int issued = prefetched;
        bool ok = true;
        for (int j = prefetched; j < tiles && ok; ++j) {
            // The raw stage is refilled as soon as the split warps have converted it (the MMAs
            // read only the converted layouts); j >= kStages here.
            ok = mbar_wait(&s.raw_free[j % kStages], ((j / kStages) - 1) & 1);
            if (!ok) break;
            issue(j);
            ++issued;
        }
        if (!ok) {
            for (int j = max(0, issued - kStages); j < issued; ++j) mbar_wait(&s.full[j % kStages], (j / kStages) & 1);
        }
        // Prefetched tiles past the visited ones: converted for nothing; wait for their loads.
        for (int j = tiles; j < prefetched; ++j) mbar_wait(&s.full[j], 0);
    }
}

// Split warps (two, 64 threads; w = 0 or 1): FP16 conversion of each column tile and its column
// statistics.
template <int D, bool kKeyRows, class St>
__device__ __forceinline__ void split_role(St &s, const AttentionParams &p, const TileWindow &t, int w, int lane) {
    constexpr int kStages = St::kStages;
    const int first = t.first, last = t.last, window_tiles = t.window_tiles, prefetched = t.prefetched;
    const long long query_base = t.query_base;
    const unsigned char *mask = t.mask;
    const auto visible_tiles = [&]() { return visited_tiles(s); };
    // Split warp w owns rows [32w, 32w + 32) of each column tile for the maxima, the masks and
    // the column statistics; convert_stage writes the operand layouts.
    const int row = 32 * w + lane;
    const float scale1 = kKeyRows ? p.scale : 1.f;  // Q enters the products as scale * Q
    // This lane's column statistics (key rows: the query's saved {max, sum} and delta; query
    // rows: whether the key exists and is visible), loaded one tile ahead so that their global
    // load latency overlaps the previous tile's conversion.
    float next_max = -INFINITY, next_total = 0.f, next_delta = 0.f;
    bool next_flag = false;
    const auto load_stats = [&](int jj) {
        const int column = first + jj * kCols + row;
        next_flag = jj < window_tiles && column < last;
        if (kKeyRows) {
            next_max = next_flag ? p.lse_in[(query_base + column) * 2] : -INFINITY;
            next_total = next_flag ? p.lse_in[(query_base + column) * 2 + 1] : 0.f;
            next_delta = next_flag ? p.delta[query_base + column] : 0.f;
        } else {
            next_flag = next_flag && mask[column] != 0;
        }
    };
    load_stats(0);
    // Query rows: the prefetched tiles are converted without waiting for the visited-tile
    // count (which comes from a mask read); those past it are converted for nothing and never
    // consumed. Key rows (count 0 or the whole window) wait for it.
    int tiles = kKeyRows ? __shfl_sync(0xffffffffu, visible_tiles(), 0) : prefetched;
    bool counted = kKeyRows;
    for (int j = 0; j < tiles || !counted; ++j) {
        if (!counted && j >= prefetched) {
            tiles = __shfl_sync(0xffffffffu, visible_tiles(), 0);
            counted = true;
            if (j >= tiles) break;
        }
        const int stage = j % kStages, parity = j & 1;
        const float maximum = next_max, total = next_total, delta = next_delta;
        const bool flag = next_flag;
        load_stats(j + 1);
        const bool landed = __all_sync(0xffffffffu, mbar_wait(&s.full[stage], (j / kStages) & 1));
        if (lane == 0) RK_BTRACE(j, 1 + w);
        bool visible;
        float delta_abs = 0.f, col_offset = -INFINITY;
        if (kKeyRows) {  // column = query: visible if it exists and has a finite row max
            visible = flag && maximum != -INFINITY;
            col_offset = visible ? 14.f - maximum * kLog2e - __log2f(total) : -INFINITY;
            delta_abs = visible ? fabsf(delta) : 0.f;
        } else {  // column = key: visible if it exists and is not masked
            visible = flag;
        }
        const uint32_t bits = __ballot_sync(0xffffffffu, visible);
        // Rows of masked key columns are zeroed (query rows only).
        const bool keep_row = kKeyRows || ((bits >> lane) & 1);
        float max1 = 0.f, max2 = 0.f;
#pragma unroll
        for (int c = 0; c < D / 4; ++c) {
            const float4 x = raw_chunk<D>(s.raw1[stage], row, c);
            const float4 y = raw_chunk<D>(s.raw2[stage], row, c);
            if (keep_row) {
                max1 = max3(max1, fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w)));
                max2 = max3(max2, fmaxf(fabsf(y.x), fabsf(y.y)), fmaxf(fabsf(y.z), fabsf(y.w)));
            }
        }
#pragma unroll
        for (int offset = 16; offset; offset >>= 1) {
            max1 = fmaxf(max1, __shfl_xor_sync(0xffffffffu, max1, offset));
            max2 = fmaxf(max2, __shfl_xor_sync(0xffffffffu, max2, offset));
            delta_abs = fmaxf(delta_abs, __shfl_xor_sync(0xffffffffu, delta_abs, offset));
        }
        // The stage's statistics and converted layouts (read by the row warps and the MMAs
        // for tile j - kStages) are rewritten only after those MMAs finished.
        const bool stage_free = j < kStages || __all_sync(0xffffffffu, mbar_wait(&s.empty[stage], ((j / kStages) - 1) & 1));
        if (kKeyRows) {
            s.col_offset[stage][row] = col_offset;
            s.col_delta[stage][row] = delta;
        }
        if (lane == 0) {
            s.split_max[parity][w][0] = max1;
            s.split_max[parity][w][1] = max2;
            s.split_max[parity][w][2] = delta_abs;
            s.split_ok[parity][w] = landed && stage_free;
            s.col_mask[stage][w] = bits;
        }
        // One barrier per tile: the maxima are double-buffered by tile parity.
        asm volatile("bar.sync 1, 64;" ::: "memory");
        if (!(s.split_ok[parity][0] && s.split_ok[parity][1])) break;
        const int e1 = fp16_scale_exponent(fmaxf(s.split_max[parity][0][0], s.split_max[parity][1][0]) * scale1);
        const int e2 = fp16_scale_exponent(fmaxf(s.split_max[parity][0][1], s.split_max[parity][1][1]));
        if (w == 0 && lane == 0) {
            s.e1[stage] = e1;
            s.e2[stage] = e2;
            s.col_delta_max[stage] = fmaxf(s.split_max[parity][0][2], s.split_max[parity][1][2]);
        }
        convert_stage<D>(s, stage, w, lane, keep_row, exp2_int(e1) * scale1, exp2_int(e2));
        mbar_arrive(&s.raw_free[stage]);
        fence_proxy_async_shared();
        if (lane == 0) RK_BTRACE(j, 3 + w);
        mbar_arrive(&s.ready[stage]);
    }
}

template <int D, bool kKeyRows>
__global__ void __launch_bounds__(kThreads, Geometry<D>::kCtasPerSm)
        backward_kernel(const BackwardArgs args, const __grid_constant__ CUtensorMap tmap1,
                        const __grid_constant__ CUtensorMap tmap2) {
    using G = Geometry<D>;
    using C = Columns<D, kKeyRows>;
    using S = Storage<D, kKeyRows>;
    constexpr int kStages = S::kStages;
    extern __shared__ uint8_t shared_raw[];
    S &s = *reinterpret_cast<S *>((reinterpret_cast<uintptr_t>(shared_raw) + 1023) & ~uintptr_t(1023));
    const AttentionParams &p = args.p;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    const TileWindow window = tile_window<kStages>(p, kKeyRows, args.blocks_per_head);
    const int h = window.h, b = window.b, r0 = window.r0, row_count = window.row_count, first = window.first;
    const long long query_base = window.query_base;
    const long long key_base = (static_cast<long long>(b) * p.heads + h) * p.keys;
    const unsigned char *mask = window.mask;

    if (warp == 0) {
        tmem_alloc(&s.tmem_base, G::kTmemColumns);
        tmem_relinquish();
    }
    if (threadIdx.x == kProducerWarp * 32) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.raw_free[i], kSplitThreads);
            mbar_init(&s.ready[i], kSplitThreads);
            mbar_init(&s.empty[i], 1);
        }
        mbar_init(&s.s_full, 1);
        mbar_init(&s.p_full, kRows);
        mbar_init(&s.x_done, 1);
        mbar_init(&s.rows_ready, kRows);
        mbar_init(&s.range_ready, 1);
        mbar_init(&s.mma_done, 1);
        mbar_fence_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s.tmem_base;

    if (warp == kProducerWarp) {
        // ---------------------------------------------------------------- TMA producer
        producer_role<D, kKeyRows>(s, window, tmap1, tmap2, lane);
    } else if (warp == kMmaWarp) {
        // ---------------------------------------------------------------- MMA issuer
        const int tiles = __shfl_sync(0xffffffffu, visited_tiles(s), 0);
        if (tiles > 0) {
            constexpr uint64_t row_stage = G::kRowWords * 4 / 16;
            const uint64_t b1_desc = sw128_descriptor(smem_u32(s.b1[0]));
            const uint64_t b2_desc = sw128_descriptor(smem_u32(s.b2[0]));
            const uint64_t b1_mn_desc = sw128_mn_descriptor(smem_u32(s.b1[0]), G::kMnChunkBytes);
            const uint64_t b2_mn_desc = sw128_mn_descriptor(smem_u32(s.b2[0]), G::kMnChunkBytes);
            bool ok = mbar_wait_warp(&s.rows_ready, 0);
            for (int j = 0; j < tiles && ok; ++j) {
                const int stage = j % kStages;
                ok = mbar_wait_warp(&s.ready[stage], (j / kStages) & 1);
                if (!ok) break;
                tc_fence_after();
                if constexpr (C::kRowOperandsInSmem) {
                    issue_product_smem<D>(tmem + C::kS, sw128_descriptor(smem_u32(s.a.a1)), b1_desc + row_stage * stage, nullptr);
                    if (lane == 0) RK_BTRACE(j, 4);
                    issue_product_smem<D>(tmem + C::kDP, sw128_descriptor(smem_u32(s.a.a2)), b2_desc + row_stage * stage, &s.s_full);
                } else {
                    issue_product<D>(tmem + C::kS, tmem + C::kA1, b1_desc + row_stage * stage, nullptr);
                    if (lane == 0) RK_BTRACE(j, 4);
                    issue_product<D>(tmem + C::kDP, tmem + C::kA2, b2_desc + row_stage * stage, &s.s_full);
                }
                ok = mbar_wait_warp(&s.p_full, j & 1);
                if (lane == 0) RK_BTRACE(j, 5);
                if (!ok) break;
                tc_fence_after();
                if constexpr (kKeyRows) {
                    issue_x<D>(tmem + C::kX1, tmem + C::kDP, b1_mn_desc + row_stage * stage, nullptr);
                    issue_x<D>(tmem + C::kX2, tmem + C::kS, b2_mn_desc + row_stage * stage, &s.x_done);
                } else {
                    issue_x<D>(tmem + C::kX1, tmem + C::kDP, b1_mn_desc + row_stage * stage, &s.x_done);
                }
                mma_commit_warp(&s.empty[stage]);
            }
            mma_commit_warp(&s.mma_done);
            mbar_wait_warp(&s.mma_done, 0);
        }
    } else if (warp >= kSplitWarp) {
        // ---------------------------------------------------------------- FP16 split
        split_role<D, kKeyRows>(s, p, window, warp - kSplitWarp, lane);
    } else {
        // ---------------------------------------------------------------- row warps
        const int r = threadIdx.x;  // row within the tile = TMEM lane
        const int row = r0 + r;
        const bool row_valid = row < row_count;
        const uint32_t lanes = lane_address(tmem, warp);
        bool row_active;  // the row takes part at all (query: finite max; key: visible)
        float row_offset = -INFINITY, row_delta = 0.f, row_l1 = 0.f;
        int ea1, ea2;
        {
            float x[D];
            if (kKeyRows) {
                row_active = row_valid && mask[row] != 0;
                load_row<D>(p.v.row(b, h, row_valid ? row : 0), row_active, 1.f, x);
#pragma unroll
                for (int c = 0; c < D; ++c) row_l1 += fabsf(x[c]);
                ea2 = fp16_scale_exponent(abs_max<D>(x));
                if constexpr (C::kRowOperandsInSmem)
                    store_row_operand_smem<D>(x, ea2, s.a.a2, r);
                else
                    store_row_operand<D>(x, ea2, lanes + C::kA2);
                load_row<D>(p.k.row(b, h, row_valid ? row : 0), row_active, 1.f, x);
            } else {
                const float maximum = row_valid ? p.lse_in[(query_base + row) * 2] : -INFINITY;
                const float total = row_valid ? p.lse_in[(query_base + row) * 2 + 1] : 0.f;
                row_active = row_valid && maximum != -INFINITY;
                if (row_active) row_offset = 14.f - maximum * kLog2e - __log2f(total);
                load_row<D>(p.dout.row(b, h, row_valid ? row : 0), row_valid, 1.f, x);
                const float4 *o4 = reinterpret_cast<const float4 *>(p.o_in.row(b, h, row_valid ? row : 0));
                float delta = 0.f;
#pragma unroll
                for (int c = 0; c < D / 4; ++c) {
                    const float4 o = row_valid ? __ldg(o4 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
                    delta = fmaf(x[4 * c], o.x, delta);
                    delta = fmaf(x[4 * c + 1], o.y, delta);
                    delta = fmaf(x[4 * c + 2], o.z, delta);
                    delta = fmaf(x[4 * c + 3], o.w, delta);
                }
#pragma unroll
                for (int c = 0; c < D; ++c) row_l1 += fabsf(x[c]);
                row_delta = delta;
                if (row_valid) p.delta[query_base + row] = delta;
                ea2 = fp16_scale_exponent(abs_max<D>(x));
                store_row_operand<D>(x, ea2, lanes + C::kA2);
                load_row<D>(p.q.row(b, h, row_valid ? row : 0), row_valid, p.scale, x);
            }
            ea1 = fp16_scale_exponent(abs_max<D>(x));
            if constexpr (C::kRowOperandsInSmem) {
                store_row_operand_smem<D>(x, ea1, s.a.a1, r);
                fence_proxy_async_shared();  // the stores, visible to the MMAs' shared-memory reads
            } else {
                store_row_operand<D>(x, ea1, lanes + C::kA1);
            }
            tc_fence_before();
            mbar_arrive(&s.rows_ready);
        }

        float acc1[D], acc2[kKeyRows ? D : 1];
#pragma unroll
        for (int c = 0; c < D; ++c) acc1[c] = 0.f;
#pragma unroll
        for (int c = 0; c < (kKeyRows ? D : 1); ++c) acc2[c] = 0.f;
        float pending_scale1 = 0.f, pending_scale2 = 0.f;  // 2^-(scales) of the last tile's X1, X2
        bool ok = true;
        const int tiles = __shfl_sync(0xffffffffu, visited_tiles(s), 0);
        for (int j = 0; j < tiles && ok; ++j) {
            const int stage = j % kStages;
            ok = __all_sync(0xffffffffu, mbar_wait(&s.s_full, j & 1) && mbar_wait(&s.ready[stage], (j / kStages) & 1));
            if (lane == 0 && (warp == 0 || warp == 3)) RK_BTRACE(j, warp == 0 ? 6 : 9);
            if (!ok) break;
            tc_fence_after();
            const int c0 = first + j * kCols;
            const int e1 = s.e1[stage], e2 = s.e2[stage];
            const float slope = kLog2e * exp2_int(-(ea1 + e1));  // TMEM S -> log2e * score
            const float dp_scale = exp2_int(-(ea2 + e2));        // TMEM dP -> dP
            // |dS| <= ||row operand 2||_1 * max|column operand 2| + |delta| (P <= 1)
            const float bound = row_l1 * exp2_int(15 - e2) + (kKeyRows ? s.col_delta_max[stage] : fabsf(row_delta));
            const int g = fp16_scale_exponent(bound);
            const float to_ds = exp2_int(g - 14);  // P' (= 2^14 P) * (dP - delta) * to_ds = 2^g dS
            const float w_scale = dp_scale * to_ds;
            uint64_t active = row_active ? (static_cast<uint64_t>(s.col_mask[stage][0]) |
                                            (static_cast<uint64_t>(s.col_mask[stage][1]) << 32))
                                         : 0ull;
            if (p.radius >= 0) {
                const int lo_col = max(0, row - p.radius - c0), hi_col = min(kCols - 1, row + p.radius - c0);
                active &= lo_col > hi_col ? 0ull : ((~0ull) >> (63 - (hi_col - lo_col))) << lo_col;
            }
            const bool all_active = __all_sync(0xffffffffu, active == ~0ull);
#pragma unroll 1
            for (int chunk = 0; chunk < 4; ++chunk) {  // rolled: keeps one chunk's values live
                float sv[16], dv[16];  // scores, then P'; dP, then dS'
                tmem_load16x2(lanes + C::kS + 16 * chunk, sv, lanes + C::kDP + 16 * chunk, dv);
                // key rows, d = 32: the chunk's 16 query statistics with 16-byte loads (d = 64 keeps
                // scalar loads: its key-rows kernel is at the register limit)
                float col_offset[16], col_delta[16];
                if constexpr (kKeyRows && D == 32) {
                    const float4 *o4 = reinterpret_cast<const float4 *>(&s.col_offset[stage][16 * chunk]);
                    const float4 *d4 = reinterpret_cast<const float4 *>(&s.col_delta[stage][16 * chunk]);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float4 o = o4[i], d = d4[i];
                        col_offset[4 * i] = o.x, col_offset[4 * i + 1] = o.y, col_offset[4 * i + 2] = o.z, col_offset[4 * i + 3] = o.w;
                        col_delta[4 * i] = d.x, col_delta[4 * i + 1] = d.y, col_delta[4 * i + 2] = d.z, col_delta[4 * i + 3] = d.w;
                    }
                }
                // Column pairs as packed FP32 pairs (fma/mul .f32x2), except in the d = 32
                // key-rows kernel, whose 128 registers a thread cannot hold the pairs.
                if constexpr (kKeyRows && D == 32) {
#pragma unroll
                    for (int c = 0; c < 16; ++c) {
                        const int col = 16 * chunk + c;
                        const float offset = !kKeyRows ? row_offset : D == 32 ? col_offset[c] : s.col_offset[stage][col];
                        const float delta = !kKeyRows ? row_delta : D == 32 ? col_delta[c] : s.col_delta[stage][col];
                        float pv = fast_exp2(fmaf(sv[c], slope, offset));
                        if (!all_active) pv = (active >> col) & 1 ? pv : 0.f;
                        sv[c] = pv;
                        dv[c] = pv * fmaf(dv[c], w_scale, -delta * to_ds);
                    }
                } else {
#pragma unroll
                    for (int c = 0; c < 16; c += 2) {  // column pairs as packed FP32 pairs
                        const int col = 16 * chunk + c;
                        float2 offset, delta;
                        if constexpr (!kKeyRows) {
                            offset = make_float2(row_offset, row_offset);
                            delta = make_float2(row_delta, row_delta);
                        } else if constexpr (D == 32) {
                            offset = make_float2(col_offset[c], col_offset[c + 1]);
                            delta = make_float2(col_delta[c], col_delta[c + 1]);
                        } else {
                            offset = make_float2(s.col_offset[stage][col], s.col_offset[stage][col + 1]);
                            delta = make_float2(s.col_delta[stage][col], s.col_delta[stage][col + 1]);
                        }
                        const float2 arg = fma_f32x2(make_float2(sv[c], sv[c + 1]), make_float2(slope, slope), offset);
                        float pa = fast_exp2(arg.x), pb = fast_exp2(arg.y);
                        if (!all_active) {
                            pa = (active >> col) & 1 ? pa : 0.f;
                            pb = (active >> (col + 1)) & 1 ? pb : 0.f;
                        }
                        sv[c] = pa;
                        sv[c + 1] = pb;
                        // dS' = P' (dP w - delta to_ds)
                        const float2 shifted = fma_f32x2(make_float2(dv[c], dv[c + 1]), make_float2(w_scale, w_scale),
                                                         mul_f32x2(delta, make_float2(-to_ds, -to_ds)));
                        const float2 ds = mul_f32x2(make_float2(pa, pb), shifted);
                        dv[c] = ds.x;
                        dv[c + 1] = ds.y;
                    }
                }
                store_split_chunk(lanes + C::kDP + 16 * chunk, dv);
                if (kKeyRows) store_split_chunk(lanes + C::kS + 16 * chunk, sv);
            }
            if (lane == 0 && warp == 0) RK_BTRACE(j, 11);
            // Fold the previous tile's X before the P(j)/dS(j) arrival lets the MMA warp
            // overwrite it.
            if (j > 0) {
                ok = __all_sync(0xffffffffu, mbar_wait(&s.x_done, (j - 1) & 1));
                if (!ok) {
                    tmem_wait_store();
                    break;
                }
                tc_fence_after();
                fold_x<D, kKeyRows>(acc1, acc2, lanes, pending_scale1, pending_scale2);
            }
            if (lane == 0 && warp == 0) RK_BTRACE(j, 8);
            tmem_wait_store();
            tc_fence_before();
            if (lane == 0 && (warp == 0 || warp == 3)) RK_BTRACE(j, warp == 0 ? 7 : 10);
            mbar_arrive(&s.p_full);
            // X1 = 2^(g + e1) * (dS . column operand 1); X2 = 2^(14 + e2) * (P . dO)
            pending_scale1 = exp2_int(-(g + e1));
            pending_scale2 = exp2_int(-(14 + e2));
        }
        if (tiles > 0 && ok) {
            ok = __all_sync(0xffffffffu, mbar_wait(&s.x_done, (tiles - 1) & 1));
            tc_fence_after();
            if (ok) fold_x<D, kKeyRows>(acc1, acc2, lanes, pending_scale1, pending_scale2);
        }
        // Outputs (packed [batch][heads][tokens][D]); a failed wait leaves NaN.
        if (row_valid) {
            const float bad = ok ? 1.f : NAN;
            if constexpr (kKeyRows) {
                float4 *dk = reinterpret_cast<float4 *>(p.dk + (key_base + row) * D);
                float4 *dv = reinterpret_cast<float4 *>(p.dv + (key_base + row) * D);
#pragma unroll
                for (int c = 0; c < D / 4; ++c) {
                    if (row_active) {
                        dk[c] = make_float4(acc1[4 * c] * bad, acc1[4 * c + 1] * bad, acc1[4 * c + 2] * bad, acc1[4 * c + 3] * bad);
                        dv[c] = make_float4(acc2[4 * c] * bad, acc2[4 * c + 1] * bad, acc2[4 * c + 2] * bad, acc2[4 * c + 3] * bad);
                    } else {
                        dk[c] = dv[c] = make_float4(0.f, 0.f, 0.f, 0.f);  // masked key: exactly zero
                    }
                }
            } else {
                float4 *dq = reinterpret_cast<float4 *>(p.dq + (query_base + row) * D);
                const float scale = p.scale * bad;
#pragma unroll
                for (int c = 0; c < D / 4; ++c)
                    dq[c] = make_float4(acc1[4 * c] * scale, acc1[4 * c + 1] * scale, acc1[4 * c + 2] * scale, acc1[4 * c + 3] * scale);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, G::kTmemColumns);
    }
}

// ---- fused single-pass backward (d = 32) ---------------------------------------------------------
// One key-major pass computes dK, dV and dQ: the key-rows kernel's S^T, dP^T, P and dS^T, plus
// dQ = scale dS K per 64-query tile as a tensor-core product whose A is dS^T from shared memory
// (MN-major: each key row's 64 query values are one 128-byte row) and whose B is the CTA's K rows
// read MN-major ([k0 | k1], N = 64). The per-tile dQ rows are added into the gradient with FP32
// atomics (the summation order over key tiles is not fixed). K and dS enter that product with one
// exponent for all 128 keys of the CTA (the key-rows pass scales them per key).
//
// A column pre-pass runs first, once per 64-query tile: it writes delta, zeroes dQ, and stores in
// the caller's workspace the tile's operands already split -- scale Q and dO as FP16 rows
// [x0 | x1] (128 bytes per query, the row layout the key-rows pass builds in its split warps for
// every key tile again) -- and a record of the tile's column statistics (exponents, softmax
// offsets, delta). The main kernel TMA-loads those tiles straight into the operand layout (a 128B-
// swizzled box of 64 FP16 x 64 rows) and has no split warps: one CTA per SM (512 TMEM columns),
// warps 0-7 two row warpgroups -- warpgroup g handles columns [32 g, 32 g + 32) of every tile and
// features [16 g, 16 g + 16) of the outputs -- warp 8 the TMA producer, warp 9 the issuer of the
// S^T, dP^T, dK and dV products, warp 10 the issuer of the dQ products (two issuing warps on two
// sub-partitions; both wait for the row warps with suspending waits, so that they take no issue
// slots from the row warps beside them). S and dP are double-buffered so that the next tile's
// products run while the row warps work on this one; the row warps fold a tile's dK, dV and dQ
// products while they work on the next. Query tiles are 64-aligned (the window's first tile
// starts at a multiple of 64; the radius test zeroes the columns outside the window).
namespace fused {
constexpr int kThreads = 352;
constexpr int kRowThreads = 256;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;    // S, dP, dK and dV products
constexpr int kDqWarp = 10;    // dQ products (a second issuing warp, on another sub-partition)
// TMEM columns: S / P and dP / dS of tile parity i at 128 i and 128 i + 64; X1 (dK) and X2 (dV)
// as [b0 | b1] products; dQ (M = 64: query m at lane (m % 16) + 32 (m / 16)) as [k0 | k1].
constexpr uint32_t kScores = 0, kX1 = 256, kX2 = 320, kDQ = 384;
constexpr uint32_t kTmemColumns = 512;
// dQ: M = 64, N = 64, A and B both MN-major.
constexpr uint32_t kIdescDQ = f16_instr_desc(64, 64) | (1u << 15) | (1u << 16);

// Column statistics of one 64-query tile, written by the pre-pass.
struct alignas(16) TileRecord {
    float col_offset[kCols];  // 14 - max log2e - log2(sum) per query; -inf if it sees no key (or does not exist)
    float col_delta[kCols];   // delta per visible query, else 0
    int e1, e2;               // exponents of the tile's scale Q and dO splits
    float delta_max;          // max |col_delta|
    int unused;
};
constexpr uint32_t kRecordBytes = sizeof(TileRecord);
static_assert(kRecordBytes % 16 == 0, "bulk copies move multiples of 16 bytes");
constexpr uint32_t kTileBytes = kCols * 128;  // one split tile: 64 rows x [x0 | x1] FP16

// Workspace carve-up for B*H*Q queries: split Q rows, split dO rows (each padded to 64 queries per
// (batch, head)), then the tile records. Offsets in bytes, all 16-byte aligned.
struct Workspace {
    long long tiles_per_head, rows, q_offset, dout_offset, record_offset, bytes;
};
__host__ __device__ inline Workspace workspace_layout(long long batch_heads, long long queries) {
    Workspace w;
    w.tiles_per_head = (queries + kCols - 1) / kCols;
    w.rows = batch_heads * w.tiles_per_head * kCols;
    w.q_offset = 0;
    w.dout_offset = w.rows * 128;
    w.record_offset = 2 * w.rows * 128;
    w.bytes = w.record_offset + batch_heads * w.tiles_per_head * kRecordBytes;
    return w;
}

struct alignas(1024) Storage {
    static constexpr int kStages = 4;
    uint32_t b1[kStages][kCols * 32];        // scale Q rows as split FP16 [q0 | q1] (B of S^T; MN-major B of dK), 128B swizzle
    uint32_t b2[kStages][kCols * 32];        // dO rows (B of dP^T; MN-major B of dV)
    uint32_t a1[kRows * 32];                 // K rows [k0 | k1] (A of S^T; MN-major B of dQ)
    uint32_t a2[kRows * 32];                 // V rows (A of dP^T)
    uint32_t ds[2][2][kRows * 32];           // [tile parity][term]: dS^T rows, 64 FP16 queries per key (A of dQ)
    TileRecord record[kStages];
    float row_max[4][2];                     // per row warp of warpgroup 0: max |K|, max ||V row||_1
    uint64_t full[kStages];                  // the stage's tiles and record landed (TMA bytes)
    uint64_t empty[kStages];                 // MMAs reading the stage finished (commit)
    uint64_t s_full[2];                      // S and dP of the tile parity in TMEM (commit)
    uint64_t p_full;                         // P / dS stored, the previous products folded (256 arrivals)
    uint64_t x_done;                         // dK, dV and dQ products of the tile in TMEM (two commits)
    uint64_t rows_ready;                     // K and V rows stored (256 arrivals)
    uint64_t mma_done;
    uint64_t dq_done;
    uint64_t range_ready;
    uint32_t tmem_base;
    int tile_count;
};

constexpr int shared_bytes() { return static_cast<int>(sizeof(Storage)) + 1024; }
static_assert(shared_bytes() <= 227 * 1024, "fused backward: shared memory");

struct Args {
    AttentionParams p;
    int blocks_per_head;  // key tiles per (batch, head)
    long long tiles_per_head;  // 64-query tiles per (batch, head) in the workspace
    const TileRecord *records;
};

// store_split_chunk, also writing the two FP16 terms into the dS^T tiles of key row `row`
// (queries 16 chunk .. 16 chunk + 15 = 16-byte chunks 2 chunk and 2 chunk + 1, 128B swizzle).
__device__ __forceinline__ void store_split_chunk_dual(uint32_t column, const float (&v)[16], uint32_t *tile0, uint32_t *tile1,
                                                       int row, int chunk) {
    uint32_t q0[8], q1[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        const float x0 = __uint_as_float(__float_as_uint(v[2 * c]) & 0xFFFFE000u);
        const float y0 = __uint_as_float(__float_as_uint(v[2 * c + 1]) & 0xFFFFE000u);
        const float2 residual = sub_f32x2(make_float2(v[2 * c], v[2 * c + 1]), make_float2(x0, y0));
        q0[c] = pack_half2(x0, y0);
        q1[c] = pack_half2(residual.x, residual.y);
    }
    tmem_store8x2_async(column, reinterpret_cast<const float *>(q0), column + 8, reinterpret_cast<const float *>(q1));
    uint4 *t0 = reinterpret_cast<uint4 *>(tile0) + row * 8;
    uint4 *t1 = reinterpret_cast<uint4 *>(tile1) + row * 8;
    const int swizzle = row & 7;
    t0[(2 * chunk) ^ swizzle] = make_uint4(q0[0], q0[1], q0[2], q0[3]);
    t0[(2 * chunk + 1) ^ swizzle] = make_uint4(q0[4], q0[5], q0[6], q0[7]);
    t1[(2 * chunk) ^ swizzle] = make_uint4(q1[0], q1[1], q1[2], q1[3]);
    t1[(2 * chunk + 1) ^ swizzle] = make_uint4(q1[4], q1[5], q1[6], q1[7]);
}

// Folds a finished tile's products, the six 16-column blocks in one TMEM round trip: acc1 += X1 *
// scale1 and acc2 += X2 * scale2 for features [16 g, 16 g + 16) (warpgroup g), and that feature
// half of the tile's dQ rows added into the gradient (lanes 0-15 of warp w hold queries
// 16 (w % 4) + lane). `tile` = the gradient row of the tile's first query, `valid` = queries of
// the tile that exist.
__device__ __forceinline__ void fold_all(float (&acc1)[16], float (&acc2)[16], uint32_t lanes, int g, float scale1, float scale2,
                                         float *tile, int valid, int warp, int lane, float dq_scale) {
    float v[6][16];
    const uint32_t x = lanes + kX1 + 16 * g, y = lanes + kX2 + 16 * g, z = lanes + kDQ + 16 * g;
    const uint32_t at[6] = {x, x + 32, y, y + 32, z, z + 32};
    tmem_load16x6(at, v);
#pragma unroll
    for (int c = 0; c < 16; c += 2) {
        const float2 r1 = fma_f32x2(add_f32x2(make_float2(v[0][c], v[0][c + 1]), make_float2(v[1][c], v[1][c + 1])),
                                    make_float2(scale1, scale1), make_float2(acc1[c], acc1[c + 1]));
        const float2 r2 = fma_f32x2(add_f32x2(make_float2(v[2][c], v[2][c + 1]), make_float2(v[3][c], v[3][c + 1])),
                                    make_float2(scale2, scale2), make_float2(acc2[c], acc2[c + 1]));
        acc1[c] = r1.x;
        acc1[c + 1] = r1.y;
        acc2[c] = r2.x;
        acc2[c + 1] = r2.y;
    }
    const int m = 16 * (warp & 3) + lane;
    if (lane < 16 && m < valid) {
        float4 *dst = reinterpret_cast<float4 *>(tile + m * 32 + 16 * g);
#pragma unroll
        for (int i = 0; i < 4; ++i)
            atomicAdd(dst + i, make_float4((v[4][4 * i] + v[5][4 * i]) * dq_scale, (v[4][4 * i + 1] + v[5][4 * i + 1]) * dq_scale,
                                           (v[4][4 * i + 2] + v[5][4 * i + 2]) * dq_scale,
                                           (v[4][4 * i + 3] + v[5][4 * i + 3]) * dq_scale));
    }
}

// Column pre-pass: one CTA per 64-query tile of a (batch, head), eight threads per query (four
// features each). delta_i = sum_c dO_ic O_ic to p.delta, dQ_i = 0, and into the workspace: the
// tile's scale Q and dO rows split (scaled by 2^e1, 2^e2: the tile maxima brought into
// [2^14, 2^15)) as FP16 [x0 | x1], and its TileRecord.
constexpr int kPrepassThreads = kCols * 8;
__global__ void __launch_bounds__(kPrepassThreads) prepass_kernel(const AttentionParams p, uint8_t *workspace, long long tiles_per_head,
                                                                  long long record_offset, long long dout_offset) {
    __shared__ float maxima[kPrepassThreads / 32][3];
    const long long tile_id = blockIdx.x;
    const long long bh = tile_id / tiles_per_head;
    const int tile = static_cast<int>(tile_id % tiles_per_head);
    const int h = static_cast<int>(bh % p.heads), b = static_cast<int>(bh / p.heads);
    const int row = threadIdx.x >> 3, part = threadIdx.x & 7;
    const int query = tile * kCols + row;
    const bool valid = query < p.queries;
    const long long query_row = bh * p.queries + query;  // packed [batch][heads][queries] index
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f), u = x, o = x;
    if (valid) {
        x = __ldg(reinterpret_cast<const float4 *>(p.q.row(b, h, query)) + part);
        u = __ldg(reinterpret_cast<const float4 *>(p.dout.row(b, h, query)) + part);
        o = __ldg(reinterpret_cast<const float4 *>(p.o_in.row(b, h, query)) + part);
        x = make_float4(x.x * p.scale, x.y * p.scale, x.z * p.scale, x.w * p.scale);
        reinterpret_cast<float4 *>(p.dq + query_row * 32)[part] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float delta = fmaf(u.w, o.w, fmaf(u.z, o.z, fmaf(u.y, o.y, u.x * o.x)));
    delta += __shfl_xor_sync(0xffffffffu, delta, 1);
    delta += __shfl_xor_sync(0xffffffffu, delta, 2);
    delta += __shfl_xor_sync(0xffffffffu, delta, 4);
    const float maximum = valid ? p.lse_in[query_row * 2] : -INFINITY;
    const float total = valid ? p.lse_in[query_row * 2 + 1] : 0.f;
    const bool visible = valid && maximum != -INFINITY;
    const float col_offset = visible ? 14.f - maximum * kLog2e - __log2f(total) : -INFINITY;
    const float col_delta = visible ? delta : 0.f;
    float m1 = max3(fabsf(x.x), fabsf(x.y), fmaxf(fabsf(x.z), fabsf(x.w)));
    float m2 = max3(fabsf(u.x), fabsf(u.y), fmaxf(fabsf(u.z), fabsf(u.w)));
    float m3 = fabsf(col_delta);
#pragma unroll
    for (int offset = 16; offset; offset >>= 1) {
        m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, offset));
        m2 = fmaxf(m2, __shfl_xor_sync(0xffffffffu, m2, offset));
        m3 = fmaxf(m3, __shfl_xor_sync(0xffffffffu, m3, offset));
    }
    const int warp = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) {
        maxima[warp][0] = m1;
        maxima[warp][1] = m2;
        maxima[warp][2] = m3;
    }
    __syncthreads();
    m1 = m2 = m3 = 0.f;
#pragma unroll
    for (int w = 0; w < kPrepassThreads / 32; ++w) {
        m1 = fmaxf(m1, maxima[w][0]);
        m2 = fmaxf(m2, maxima[w][1]);
        m3 = fmaxf(m3, maxima[w][2]);
    }
    const int e1 = fp16_scale_exponent(m1), e2 = fp16_scale_exponent(m2);
    // Split rows: 32 words per query, x0 pairs in words 0-15, x1 pairs in words 16-31; this
    // thread's features 4 part .. 4 part + 3 are x0 words 2 part, 2 part + 1 and x1 words 16 + 2 part, ....
    const long long split_row = bh * tiles_per_head * kCols + tile * kCols + row;
#pragma unroll
    for (int which = 0; which < 2; ++which) {
        const float4 v = which == 0 ? x : u;
        const float scale = exp2_int(which == 0 ? e1 : e2);
        uint32_t a0, a1, c0, c1;
        split_pack2<false>(v.x, v.y, scale, a0, a1);
        split_pack2<false>(v.z, v.w, scale, c0, c1);
        uint32_t *dst = reinterpret_cast<uint32_t *>(workspace + (which == 0 ? 0 : dout_offset)) + split_row * 32;
        *reinterpret_cast<uint2 *>(dst + 2 * part) = make_uint2(a0, c0);
        *reinterpret_cast<uint2 *>(dst + 16 + 2 * part) = make_uint2(a1, c1);
    }
    TileRecord *record = reinterpret_cast<TileRecord *>(workspace + record_offset) + tile_id;
    if (part == 0) {
        record->col_offset[row] = col_offset;
        record->col_delta[row] = col_delta;
        if (valid) p.delta[query_row] = delta;
    }
    if (threadIdx.x == 0) {
        record->e1 = e1;
        record->e2 = e2;
        record->delta_max = m3;
        record->unused = 0;
    }
}

__global__ void __launch_bounds__(kThreads, 1)
        backward_kernel(const Args args, const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_dout) {
    using S = Storage;
    constexpr int kStages = S::kStages;
    extern __shared__ uint8_t shared_raw[];
    S &s = *reinterpret_cast<S *>((reinterpret_cast<uintptr_t>(shared_raw) + 1023) & ~uintptr_t(1023));
    const AttentionParams &p = args.p;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    int block = blockIdx.x;
    const int key_tile = block % args.blocks_per_head;
    block /= args.blocks_per_head;
    const int h = block % p.heads, b = block / p.heads;
    const long long bh = static_cast<long long>(b) * p.heads + h;
    const int r0 = key_tile * kRows;
    int first, last;  // queries that can see the key tile
    key_window(r0, min(r0 + kRows, p.keys), p.queries, p.radius, first, last);
    first &= ~(kCols - 1);
    const int window_tiles = last > first ? (last - first + kCols - 1) / kCols : 0;
    const unsigned char *mask = p.mask + static_cast<long long>(b) * p.keys;

    if (warp == 0) {
        tmem_alloc(&s.tmem_base, kTmemColumns);
        tmem_relinquish();
    }
    if (threadIdx.x == kProducerWarp * 32) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.empty[i], 1);
        }
        mbar_init(&s.s_full[0], 1);
        mbar_init(&s.s_full[1], 1);
        mbar_init(&s.p_full, kRowThreads);
        mbar_init(&s.x_done, 2);
        mbar_init(&s.rows_ready, kRowThreads);
        mbar_init(&s.range_ready, 1);
        mbar_init(&s.mma_done, 1);
        mbar_init(&s.dq_done, 1);
        mbar_fence_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s.tmem_base;

    if (warp == kProducerWarp) {
        // ---------------------------------------------------------------- TMA producer
        // Tiles of the window, none when every key of the tile is masked (dK = dV = 0).
        bool visible = false;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int key = r0 + 4 * lane + e;
            visible = visible || (key < p.keys && mask[key] != 0);
        }
        const int tiles = __any_sync(0xffffffffu, visible) ? window_tiles : 0;
        if (lane == 0) {
            s.tile_count = tiles;
            mbar_arrive(&s.range_ready);
            const int row_base = static_cast<int>(bh * args.tiles_per_head * kCols) + first;
            const TileRecord *records = args.records + bh * args.tiles_per_head + first / kCols;
            bool ok = true;
            int issued = 0;
            for (int j = 0; j < tiles; ++j) {
                const int stage = j % kStages;
                if (j >= kStages && !(ok = mbar_wait(&s.empty[stage], ((j / kStages) - 1) & 1))) break;
                RK_FTRACE(j, 0);
                mbar_arrive_expect_tx(&s.full[stage], 2 * kTileBytes + kRecordBytes);
                tma_load_2d(s.b1[stage], &tmap_q, &s.full[stage], 0, row_base + j * kCols);
                tma_load_2d(s.b2[stage], &tmap_dout, &s.full[stage], 0, row_base + j * kCols);
                bulk_load(&s.record[stage], records + j, kRecordBytes, &s.full[stage]);
                ++issued;
            }
            // Every load issued lands before the CTA exits (a failed wait above ends the loop early).
            if (!ok)
                for (int j = max(0, issued - kStages); j < issued; ++j) mbar_wait(&s.full[j % kStages], (j / kStages) & 1);
        }
    } else if (warp == kMmaWarp) {
        // ---------------------------------------------------------------- MMA issuer
        // Per tile j: S(j + 1) and dP(j + 1) go out before waiting for P(j) / dS(j); then dK and
        // dV of tile j. The MMAs of one thread run in issue order, so S(j + 2) overwrites the
        // buffers of tile j only after the products that read them.
        const int tiles = __shfl_sync(0xffffffffu, visited_tiles(s), 0);
        if (tiles > 0) {
            using G = Geometry<32>;
            constexpr uint64_t row_stage = G::kRowWords * 4 / 16;
            const uint64_t b1_desc = sw128_descriptor(smem_u32(s.b1[0]));
            const uint64_t b2_desc = sw128_descriptor(smem_u32(s.b2[0]));
            const uint64_t b1_mn_desc = sw128_mn_descriptor(smem_u32(s.b1[0]), G::kMnChunkBytes);
            const uint64_t b2_mn_desc = sw128_mn_descriptor(smem_u32(s.b2[0]), G::kMnChunkBytes);
            const uint64_t k_desc = sw128_descriptor(smem_u32(s.a1));
            const uint64_t v_desc = sw128_descriptor(smem_u32(s.a2));
            const auto issue_scores = [&](int j) -> bool {
                const int stage = j % kStages;
                if (!mbar_wait_warp(&s.full[stage], (j / kStages) & 1)) return false;
                tc_fence_after();
                const uint32_t scores = tmem + kScores + 128 * (j & 1);
                issue_product_smem<32>(scores, k_desc, b1_desc + row_stage * stage, nullptr);
                issue_product_smem<32>(scores + 64, v_desc, b2_desc + row_stage * stage, &s.s_full[j & 1]);
                if (lane == 0) RK_FTRACE(j, 4);
                return true;
            };
            bool ok = mbar_wait_warp(&s.rows_ready, 0) && issue_scores(0);
            for (int j = 0; j < tiles && ok; ++j) {
                const int stage = j % kStages;
                if (j + 1 < tiles && !issue_scores(j + 1)) {
                    ok = false;
                    break;
                }
                ok = __all_sync(0xffffffffu, mbar_wait_sleep(&s.p_full, j & 1));
                if (lane == 0) RK_FTRACE(j, 5);
                if (!ok) break;
                tc_fence_after();
                const uint32_t scores = tmem + kScores + 128 * (j & 1);
                issue_x<32>(tmem + kX1, scores + 64, b1_mn_desc + row_stage * stage, nullptr);
                issue_x<32>(tmem + kX2, scores, b2_mn_desc + row_stage * stage, nullptr);
                mma_commit_warp(&s.x_done);
                mma_commit_warp(&s.empty[stage]);
                if (lane == 0) RK_FTRACE(j, 12);
            }
            mma_commit_warp(&s.mma_done);
            mbar_wait_warp(&s.mma_done, 0);
        }
    } else if (warp == kDqWarp) {
        // ---------------------------------------------------------------- dQ issuer
        // dQ(j) = dS^T(j) . K once P(j) / dS(j) are stored (it reads only shared memory and
        // writes only its own accumulator, whose previous tile the row warps folded before that
        // arrival); its commit is the second arrival on x_done.
        const int tiles = __shfl_sync(0xffffffffu, visited_tiles(s), 0);
        if (tiles > 0) {
            constexpr uint64_t k_step = 2048 / 16;  // 16 K rows of an MN-major operand
            const uint64_t k_mn_desc = sw128_mn_descriptor(smem_u32(s.a1), Geometry<32>::kMnChunkBytes);
            bool ok = true;
            for (int j = 0; j < tiles && ok; ++j) {
                ok = __all_sync(0xffffffffu, mbar_wait_sleep(&s.p_full, j & 1));
                if (!ok) break;
                tc_fence_after();
#pragma unroll
                for (int term = 0; term < 2; ++term) {
                    const uint64_t ds_desc = sw128_mn_descriptor(smem_u32(s.ds[j & 1][term]), Geometry<32>::kMnChunkBytes);
#pragma unroll
                    for (int half = 0; half < 2; ++half) {
                        const uint64_t a[4] = {ds_desc + (4 * half) * k_step, ds_desc + (4 * half + 1) * k_step,
                                               ds_desc + (4 * half + 2) * k_step, ds_desc + (4 * half + 3) * k_step};
                        const uint64_t bk[4] = {k_mn_desc + (4 * half) * k_step, k_mn_desc + (4 * half + 1) * k_step,
                                                k_mn_desc + (4 * half + 2) * k_step, k_mn_desc + (4 * half + 3) * k_step};
                        mma4_f16_ss_warp(tmem + kDQ, a, bk, kIdescDQ, term == 0 && half == 0);
                    }
                }
                mma_commit_warp(&s.x_done);
            }
            mma_commit_warp(&s.dq_done);
            mbar_wait_warp(&s.dq_done, 0);
        }
    } else {
        // ---------------------------------------------------------------- row warps
        const int g = warp >> 2;                  // warpgroup: column half of each tile, feature half of the outputs
        const int r = threadIdx.x & (kRows - 1);  // key row within the tile = TMEM lane
        const int row = r0 + r;
        const bool row_valid = row < p.keys;
        const bool row_active = row_valid && mask[row] != 0;
        const uint32_t lanes = lane_address(tmem, warp);
        float l1_max;  // max over the CTA's keys of ||v_j||_1
        int ea1, ea2;  // exponents of K (one for the CTA) and of this key's V row
        {
            float x[32];
            load_row<32>(p.v.row(b, h, row_valid ? row : 0), row_active, 1.f, x);
            float l1 = 0.f;
#pragma unroll
            for (int c = 0; c < 32; ++c) l1 += fabsf(x[c]);
            ea2 = fp16_scale_exponent(abs_max<32>(x));
            if (g == 0) store_row_operand_smem<32>(x, ea2, s.a2, r);
            load_row<32>(p.k.row(b, h, row_valid ? row : 0), row_active, 1.f, x);
            float k_max = abs_max<32>(x);
#pragma unroll
            for (int offset = 16; offset; offset >>= 1) {
                k_max = fmaxf(k_max, __shfl_xor_sync(0xffffffffu, k_max, offset));
                l1 = fmaxf(l1, __shfl_xor_sync(0xffffffffu, l1, offset));
            }
            if (g == 0 && lane == 0) {
                s.row_max[warp][0] = k_max;
                s.row_max[warp][1] = l1;
            }
            asm volatile("bar.sync 2, 256;" ::: "memory");
            k_max = max3(max3(s.row_max[0][0], s.row_max[1][0], s.row_max[2][0]), s.row_max[3][0], 0.f);
            l1_max = max3(max3(s.row_max[0][1], s.row_max[1][1], s.row_max[2][1]), s.row_max[3][1], 0.f);
            ea1 = fp16_scale_exponent(k_max);
            if (g == 1) store_row_operand_smem<32>(x, ea1, s.a1, r);
            fence_proxy_async_shared();  // the stores, visible to the MMAs' shared-memory reads
            mbar_arrive(&s.rows_ready);
        }

        float acc1[16], acc2[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) acc1[c] = acc2[c] = 0.f;
        float pending1 = 0.f, pending2 = 0.f, pending_dq = 0.f;  // scales of the last tile's products
        int pending_c0 = 0;
        bool ok = true;
        const int tiles = __shfl_sync(0xffffffffu, visited_tiles(s), 0);
        float *dq_head = p.dq + bh * p.queries * 32;
        for (int j = 0; j < tiles && ok; ++j) {
            const int stage = j % kStages;
            const uint32_t scores = lanes + kScores + 128 * (j & 1);
            ok = __all_sync(0xffffffffu, mbar_wait(&s.s_full[j & 1], (j >> 1) & 1) && mbar_wait(&s.full[stage], (j / kStages) & 1));
            if (lane == 0 && (warp & 3) == 0) RK_FTRACE(j, warp == 0 ? 6 : 9);
            if (!ok) break;
            tc_fence_after();
            const TileRecord &rec = s.record[stage];
            const int c0 = first + j * kCols;
            const int e1 = rec.e1, e2 = rec.e2;
            const float slope = kLog2e * exp2_int(-(ea1 + e1));  // TMEM S -> log2e * score
            const float dp_scale = exp2_int(-(ea2 + e2));        // TMEM dP -> dP
            // One dS exponent for the CTA: |dS| <= max_j ||v_j||_1 max|dO| + max|delta| (P <= 1)
            const int gs = fp16_scale_exponent(l1_max * exp2_int(15 - e2) + rec.delta_max);
            const float to_ds = exp2_int(gs - 14);  // P' (= 2^14 P) * (dP - delta) * to_ds = 2^gs dS
            const float w_scale = dp_scale * to_ds;
            // Columns of queries that see no key have offset -inf (P = 0); the mask and the radius
            // window are applied here.
            uint64_t active = row_active ? ~0ull : 0ull;
            if (p.radius >= 0) {
                const int lo_col = max(0, row - p.radius - c0), hi_col = min(kCols - 1, row + p.radius - c0);
                active &= lo_col > hi_col ? 0ull : ((~0ull) >> (63 - (hi_col - lo_col))) << lo_col;
            }
            const bool all_active = __all_sync(0xffffffffu, static_cast<uint32_t>(active >> (32 * g)) == ~0u);
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) {
                const int chunk = 2 * g + cc;
                float sv[16], dv[16];  // scores, then P'; dP, then dS'
                tmem_load16x2(scores + 16 * chunk, sv, scores + 64 + 16 * chunk, dv);
                float col_offset[16], col_delta[16];
                const float4 *o4 = reinterpret_cast<const float4 *>(&rec.col_offset[16 * chunk]);
                const float4 *d4 = reinterpret_cast<const float4 *>(&rec.col_delta[16 * chunk]);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float4 o = o4[i], d = d4[i];
                    col_offset[4 * i] = o.x, col_offset[4 * i + 1] = o.y, col_offset[4 * i + 2] = o.z, col_offset[4 * i + 3] = o.w;
                    col_delta[4 * i] = d.x, col_delta[4 * i + 1] = d.y, col_delta[4 * i + 2] = d.z, col_delta[4 * i + 3] = d.w;
                }
#pragma unroll
                for (int c = 0; c < 16; c += 2) {
                    const int col = 16 * chunk + c;
                    const float2 arg = fma_f32x2(make_float2(sv[c], sv[c + 1]), make_float2(slope, slope),
                                                 make_float2(col_offset[c], col_offset[c + 1]));
                    float pa = fast_exp2(arg.x), pb = fast_exp2(arg.y);
                    if (!all_active) {
                        pa = (active >> col) & 1 ? pa : 0.f;
                        pb = (active >> (col + 1)) & 1 ? pb : 0.f;
                    }
                    sv[c] = pa;
                    sv[c + 1] = pb;
                    // dS' = P' (dP w - delta to_ds)
                    const float2 shifted = fma_f32x2(make_float2(dv[c], dv[c + 1]), make_float2(w_scale, w_scale),
                                                     mul_f32x2(make_float2(col_delta[c], col_delta[c + 1]), make_float2(-to_ds, -to_ds)));
                    const float2 ds = mul_f32x2(make_float2(pa, pb), shifted);
                    dv[c] = ds.x;
                    dv[c + 1] = ds.y;
                }
                store_split_chunk_dual(scores + 64 + 16 * chunk, dv, s.ds[j & 1][0], s.ds[j & 1][1], r, chunk);
                store_split_chunk(scores + 16 * chunk, sv);
            }
            if (lane == 0 && warp == 0) RK_FTRACE(j, 11);
            // Fold the previous tile's products before the P(j)/dS(j) arrival lets the MMA warp
            // overwrite them.
            if (j > 0) {
                ok = __all_sync(0xffffffffu, mbar_wait(&s.x_done, (j - 1) & 1));
                if (lane == 0 && warp == 0) RK_FTRACE(j, 13);
                if (!ok) {
                    tmem_wait_store();
                    break;
                }
                tc_fence_after();
                fold_all(acc1, acc2, lanes, g, pending1, pending2, dq_head + pending_c0 * 32, p.queries - pending_c0, warp, lane,
                         pending_dq);
            }
            if (lane == 0 && warp == 0) RK_FTRACE(j, 8);
            tmem_wait_store();
            fence_proxy_async_shared();  // the dS^T stores, visible to the dQ MMAs
            tc_fence_before();
            mbar_arrive(&s.p_full);
            if (lane == 0) RK_FTRACE(j, warp == 0 ? 7 : warp == 4 ? 10 : warp < 4 ? warp : warp == 7 ? 3 : warp + 9);
            // dK = 2^-(gs + e1) X1; dV = 2^-(14 + e2) X2; dQ = scale 2^-(gs + ea1) (dS' . K')
            pending1 = exp2_int(-(gs + e1));
            pending2 = exp2_int(-(14 + e2));
            pending_dq = p.scale * exp2_int(-(gs + ea1));
            pending_c0 = c0;
        }
        if (tiles > 0 && ok) {
            ok = __all_sync(0xffffffffu, mbar_wait(&s.x_done, (tiles - 1) & 1));
            tc_fence_after();
            if (ok)
                fold_all(acc1, acc2, lanes, g, pending1, pending2, dq_head + pending_c0 * 32, p.queries - pending_c0, warp, lane,
                         pending_dq);
        }
        // dK, dV (packed [batch][heads][keys][32]), features [16 g, 16 g + 16); a failed wait leaves NaN.
        if (row_valid) {
            const float bad = ok ? 1.f : NAN;
            const long long key_row = bh * p.keys + row;
            float4 *dk = reinterpret_cast<float4 *>(p.dk + key_row * 32 + 16 * g);
            float4 *dv = reinterpret_cast<float4 *>(p.dv + key_row * 32 + 16 * g);
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                if (row_active) {
                    dk[c] = make_float4(acc1[4 * c] * bad, acc1[4 * c + 1] * bad, acc1[4 * c + 2] * bad, acc1[4 * c + 3] * bad);
                    dv[c] = make_float4(acc2[4 * c] * bad, acc2[4 * c + 1] * bad, acc2[4 * c + 2] * bad, acc2[4 * c + 3] * bad);
                } else {
                    dk[c] = dv[c] = make_float4(0.f, 0.f, 0.f, 0.f);  // masked key: exactly zero
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemColumns);
    }
}
}  // namespace fused

// ---- host side ----------------------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 encode_function() {
    static PFN_cuTensorMapEncodeTiled_v12000 function = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *pointer = nullptr;
        cudaDriverEntryPointQueryResult query;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &pointer, cudaEnableDefault, &query) == cudaSuccess &&
            query == cudaDriverEntryPointSuccess)
            function = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(pointer);
    });
    return function;
}

// [batch][heads][tokens][D] FP32 with the given element strides; box = 32 features x 64 tokens.
bool make_tensor_map(CUtensorMap *map, const Tensor &t, int width, int batch, int heads, int tokens) {
    auto encode = encode_function();
    if (encode == nullptr) return false;
    const cuuint64_t dims[4] = {static_cast<cuuint64_t>(width), static_cast<cuuint64_t>(tokens), static_cast<cuuint64_t>(heads),
                                static_cast<cuuint64_t>(batch)};
    const cuuint64_t strides[3] = {static_cast<cuuint64_t>(t.st) * 4, static_cast<cuuint64_t>(t.sh) * 4,
                                   static_cast<cuuint64_t>(t.sb) * 4};
    const cuuint32_t box[4] = {32, static_cast<cuuint32_t>(kCols), 1, 1};
    const cuuint32_t element_strides[4] = {1, 1, 1, 1};
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float *>(t.data), dims, strides, box, element_strides,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool tma_addressable(const Tensor &t) {
    const long long limit = 1ll << 38;
    return t.st > 0 && t.sh > 0 && t.sb > 0 && t.st % 4 == 0 && t.sh % 4 == 0 && t.sb % 4 == 0 && t.st < limit &&
           t.sh < limit && t.sb < limit && (reinterpret_cast<uintptr_t>(t.data) & 15u) == 0;
}

bool rows_addressable(const Tensor &t) {
    return t.st % 4 == 0 && t.sh % 4 == 0 && t.sb % 4 == 0 && (reinterpret_cast<uintptr_t>(t.data) & 15u) == 0;
}

template <int D, bool kKeyRows>
constexpr int shared_bytes() {
    return static_cast<int>(sizeof(Storage<D, kKeyRows>)) + 1024;
}
static_assert(shared_bytes<32, false>() <= 113 * 1024 && shared_bytes<32, true>() <= 113 * 1024, "d=32: two CTAs per SM");
static_assert(shared_bytes<64, false>() <= 227 * 1024 && shared_bytes<64, true>() <= 227 * 1024, "d=64: one CTA per SM");

template <int D, bool kKeyRows>
int launch_pass(const AttentionParams &p, const CUtensorMap &map1, const CUtensorMap &map2, cudaStream_t stream) {
    cudaError_t status = prepare_kernel<backward_kernel<D, kKeyRows>>(shared_bytes<D, kKeyRows>());
    if (status != cudaSuccess) return status;
    BackwardArgs args{};
    args.p = p;
    const int rows = kKeyRows ? p.keys : p.queries;
    args.blocks_per_head = (rows + kRows - 1) / kRows;
    const unsigned blocks = static_cast<unsigned>(args.blocks_per_head) * static_cast<unsigned>(p.heads) * static_cast<unsigned>(p.batch);
    backward_kernel<D, kKeyRows><<<blocks, kThreads, shared_bytes<D, kKeyRows>(), stream>>>(args, map1, map2);
    return cudaGetLastError();
}

template <int D>
int launch_both(const AttentionParams &p, cudaStream_t stream) {
    CUtensorMap map_k, map_v, map_q, map_dout;
    if (!make_tensor_map(&map_k, p.k, D, p.batch, p.heads, p.keys) || !make_tensor_map(&map_v, p.v, D, p.batch, p.heads, p.keys) ||
        !make_tensor_map(&map_q, p.q, D, p.batch, p.heads, p.queries) ||
        !make_tensor_map(&map_dout, p.dout, D, p.batch, p.heads, p.queries))
        return kNotEligible;
    const int status = launch_pass<D, false>(p, map_k, map_v, stream);  // delta, dQ
    if (status != cudaSuccess) return status;
    return launch_pass<D, true>(p, map_q, map_dout, stream);  // dK, dV (reads delta)
}

// 2-D FP16 map of the workspace's split rows: 64 halves (128 bytes) per row, box 64 x 64 rows,
// 128B swizzle (the row layout the MMAs read).
bool make_split_map(CUtensorMap *map, void *base, long long rows) {
    auto encode = encode_function();
    if (encode == nullptr) return false;
    const cuuint64_t dims[2] = {64, static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {128};
    const cuuint32_t box[2] = {64, static_cast<cuuint32_t>(kCols)};
    const cuuint32_t element_strides[2] = {1, 1};
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base, dims, strides, box, element_strides, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The fused backward: the column pre-pass, then the key-major pass, ordered on `stream`.
int launch_fused(const AttentionParams &p, void *workspace, cudaStream_t stream) {
    const fused::Workspace w = fused::workspace_layout(static_cast<long long>(p.batch) * p.heads, p.queries);
    if (w.rows >= (1ll << 31)) return kNotEligible;  // TMA row coordinates are 32-bit
    uint8_t *base = static_cast<uint8_t *>(workspace);
    CUtensorMap map_q, map_dout;
    if (!make_split_map(&map_q, base + w.q_offset, w.rows) || !make_split_map(&map_dout, base + w.dout_offset, w.rows))
        return kNotEligible;
    cudaError_t status = prepare_kernel<fused::backward_kernel>(fused::shared_bytes());
    if (status != cudaSuccess) return status;
    const long long tiles = static_cast<long long>(p.batch) * p.heads * w.tiles_per_head;
    fused::prepass_kernel<<<static_cast<unsigned>(tiles), fused::kPrepassThreads, 0, stream>>>(p, base, w.tiles_per_head, w.record_offset,
                                                                                               w.dout_offset);
    status = cudaGetLastError();
    if (status != cudaSuccess) return status;
    fused::Args args{};
    args.p = p;
    args.blocks_per_head = (p.keys + kRows - 1) / kRows;
    args.tiles_per_head = w.tiles_per_head;
    args.records = reinterpret_cast<const fused::TileRecord *>(base + w.record_offset);
    const unsigned blocks = static_cast<unsigned>(args.blocks_per_head) * static_cast<unsigned>(p.heads) * static_cast<unsigned>(p.batch);
    fused::backward_kernel<<<blocks, fused::kThreads, fused::shared_bytes(), stream>>>(args, map_q, map_dout);
    return cudaGetLastError();
}

}  // namespace

bool backward_supported(const AttentionParams &p) {
    return tma_addressable(p.q) && tma_addressable(p.k) && tma_addressable(p.v) && tma_addressable(p.dout) &&
           rows_addressable(p.o_in) && (reinterpret_cast<uintptr_t>(p.dq) & 15u) == 0 &&
           (reinterpret_cast<uintptr_t>(p.dk) & 15u) == 0 && (reinterpret_cast<uintptr_t>(p.dv) & 15u) == 0;
}

int launch_backward(const AttentionParams &p, int head_width, cudaStream_t stream) {
    if (head_width == 32) return launch_both<32>(p, stream);
    if (head_width == 64) return launch_both<64>(p, stream);
    return kNotEligible;
}

long long fused_backward_workspace_bytes(long long batch_heads, long long queries) {
    return fused::workspace_layout(batch_heads, queries).bytes;
}

int launch_fused_backward(const AttentionParams &p, void *workspace, cudaStream_t stream) {
    if ((reinterpret_cast<uintptr_t>(workspace) & 127u) != 0) return kNotEligible;
    return launch_fused(p, workspace, stream);
}

#ifdef RK_TC_TRACE
extern "C" __attribute__((visibility("default"))) int rocmkernels_attention_backward_trace(long long *out, int capacity) {
    const int count = 2 * kTraceTiles * kTraceEvents;
    if (capacity < count) return -1;
    if (cudaMemcpyFromSymbol(out, g_bwd_trace, sizeof(long long) * count) != cudaSuccess) return -2;
    return count;
}
#endif

unsigned int read_backward_status(bool clear) {
    unsigned int value = 0;
    if (cudaMemcpyFromSymbol(&value, g_device_status, sizeof(value)) != cudaSuccess) return ~0u;
    if (clear && value != 0) {
        const unsigned int zero = 0;
        cudaMemcpyToSymbol(g_device_status, &zero, sizeof(zero));
    }
    return value;
}

}  // namespace tc
}  // namespace rk
