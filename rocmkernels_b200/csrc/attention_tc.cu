// Tensor-core flash forward for head width 32 on sm_100a: tcgen05.mma (kind::f16) with TMEM
// accumulators, TMA-staged K/V tiles, FP32 accuracy from split FP16 operands.
//
// Replaces the reference's flash forward (attention_query_flash_body, AttentionFlash32.h:23-170):
// same results (O = softmax(scale * Q K^T, masked) V, lse = {row max, exp sum}), same masking
// and radius rules, same fully-masked / NaN conventions; different machine.
//
// CTA = 256 queries as two 128-row Q tiles ("A" and "B") that share every K/V tile.
//   warps 0-3   softmax + epilogue of Q tile A (thread = query row = TMEM lane)
//   warps 4-7   softmax + epilogue of Q tile B
//   warp  8     TMA producer: raw FP32 K and V tiles of 64 keys x 32 features, 128B swizzle
//   warp  9     MMA issuer: the whole warp runs the schedule; one elected lane issues each group
//               of MMAs and its commit as a single instruction sequence
//   warps 10-11 convert each K tile to [k0 | k1] FP16 rows and each V tile to transposed
//               [v0^T ; v1^T] FP16 rows, zero masked key rows, publish the tile's key mask and
//               the two per-tile scale exponents
//
// Split FP16 operands. Every FP32 operand x is scaled by a power of two 2^e (Q: per row; K, V:
// per tile; P: 2^14) so that its largest magnitude lies in [2^14, 2^15), then split
// x' = x0 + x1 with x0 = x' cut to 11 significant bits (exactly representable in FP16) and
// x1 = FP16(x' - x0). Products keep ~22 bits:
//   S            = q0.k1 + q1.k0 + q0.k0               (M128 N64 K16 x 6; scaled by 2^(a_i + b_j))
//   [Oa|Ob|sums] = p1.[v0 ; v1 ; 1] + p0.[v0 ; v1 ; 1] (M128 N80 K16 x 8), Ot = Oa + Ob
//   (P keeps its 2^14 in Ot and in the row sums, so it cancels in O = sum Ot / sum P; the 16
//   rows of ones make the tensor core produce the row sums of P as well)
// The scales are exact powers of two and are removed in FP32 by the softmax threads.
// S is double-buffered per Q tile: the MMA warp computes S(j+2) while the softmax threads
// work on tile j, and P(j) overwrites S(j) in TMEM (as the A operand of P.V), stored in chunks
// of 16 keys as it is computed.
// Each key tile's Ot is folded into the running output in FP32 registers (O = O * exp(m_old -
// m_new) + Ot, with the running max and sum; online softmax as in AttentionFlash32.h:96-112).
// Folding in registers keeps the cross-tile sum in round-to-nearest FP32; accumulating all
// tiles in TMEM instead loses accuracy linearly in the number of tiles.
//
// TMEM (512 columns, one CTA per SM), Q tile t uses [256t, 256t + 240):
//   q0 0-15 | q1 16-31 | S/P buffer 0: 32-95 | S/P buffer 1: 96-159 | Oa 160-191 | Ob 192-223 |
//   row sums 224-239 (P in a buffer: p0 pairs in its first 32 columns, p1 pairs in the next 32)
#include "attention_tc.cuh"

#include <cudaTypedefs.h>

#include <mutex>

#include "tc_primitives.cuh"

namespace rk {
namespace tc {

namespace {

// Optional pipeline timeline (build with -DRK_TC_TRACE; compiled out otherwise): clock64 stamps
// of CTA 0 per key tile and role, read back with rocmkernels_attention_trace().
#ifdef RK_TC_TRACE
constexpr int kTraceTiles = 64, kTraceEvents = 16;
__device__ long long g_trace[kTraceTiles][kTraceEvents];
#define RK_TRACE(tile_index, event)                                                                   \
    do {                                                                                              \
        if (blockIdx.x == 0 && (tile_index) < kTraceTiles) g_trace[(tile_index)][(event)] = clock64(); \
    } while (0)
// per softmax warp, tile 5 of CTA 0: events 0 s_full seen, 1 max done, 2 exp and P stores issued,
// 3 fold done, 4 P stores complete
__device__ long long g_warp_trace[8][8];
#define RK_WARP_TRACE(tile_index, event)                                                                          \
    do {                                                                                                         \
        if (blockIdx.x == 0 && (tile_index) == 5 && (threadIdx.x & 31) == 0) g_warp_trace[threadIdx.x >> 5][(event)] = clock64(); \
    } while (0)
#else
#define RK_WARP_TRACE(tile_index, event) \
    do {                                \
    } while (0)
#define RK_TRACE(tile_index, event) \
    do {                           \
    } while (0)
#endif

constexpr int kQTile = 128;
constexpr int kQTiles = 2;
constexpr int kCtaQueries = kQTile * kQTiles;
constexpr int kKeyTile = 64;
constexpr int kD = 32;
constexpr int kStages = 4;
constexpr int kThreads = 384;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kSplitWarp = 10;
constexpr int kSplitThreads = 64;
constexpr int kTileFloats = kKeyTile * kD;  // 2048
constexpr int kTileBytes = kTileFloats * 4;  // 8 KB
constexpr int kVRows = 2 * kD + 16;          // B of P.V: v0^T, v1^T and 16 rows of ones (row sums)
constexpr int kVTileWords = kVRows * 32;     // 80 rows x 128 bytes
constexpr uint32_t kTmemColumns = 512;
constexpr uint32_t kColQ0 = 0, kColQ1 = 16, kColBuffer = 32, kBufferColumns = 64, kColO = 160, kColTile = 256;
constexpr uint32_t kColSum = kColO + 2 * kD;  // first of the 16 row-sum columns
constexpr uint32_t kIdescS = f16_instr_desc(128, 64);       // S: 64 keys
constexpr uint32_t kIdescPV = f16_instr_desc(128, kVRows);  // P.V: [v0 ; v1 ; ones] = 80 rows
constexpr float kPScale = 16384.f;                          // P is split as P * 2^14
constexpr int kNoExponent = 1000;                           // outside every clamped scale exponent

// Every tile buffer is 8 KB (64 rows x 128 bytes) and 1024-byte aligned (the 128B swizzle atom).
struct alignas(1024) SharedStorage {
    float k_raw[kStages][kTileFloats];       // FP32 K tile as TMA lands it (64 rows x 128 B, swizzled)
    float v_raw[kStages][kTileFloats];       // FP32 V tile
    uint32_t k16[kStages][kTileFloats];      // 64 key rows x 128 B: [k0 (32 fp16) | k1 (32 fp16)], K-major 128B swizzle
    uint32_t vt16[kStages][kVTileWords];     // 80 rows x 128 B: rows 0-31 v0^T, 32-63 v1^T (64 keys each, 128B
                                             // swizzle), 64-79 FP16 ones (written once)
    uint32_t key_mask[kStages][2];           // bit c: key k0 + c visible
    int k_exponent[kStages];                 // K tile scaled by 2^k_exponent
    int v_exponent[kStages];                 // V tile scaled by 2^v_exponent
    float split_max[2][2];                   // per split warp: max |K|, max |V| of its rows
    int split_ok[2];                         // per split warp: its kv_full wait succeeded
    uint64_t kv_full[kStages];               // TMA bytes landed
    uint64_t kv_ready[kStages];              // conversion done (64 arrivals)
    uint64_t kv_empty[kStages];              // MMAs reading the stage finished (commit)
    uint64_t s_full[kQTiles][2];             // S of a buffer is in TMEM (commit)
    uint64_t p_full[kQTiles];                // P of the current tile is in TMEM (128 arrivals)
    uint64_t pv_done[kQTiles];               // Ot of the current tile is in TMEM (commit)
    uint64_t q_ready;                        // q0/q1 of both tiles in TMEM (256 arrivals)
    uint64_t mma_done;                       // every MMA of the CTA finished (commit)
    uint32_t tmem_base;
};

struct FlashArgs {
    AttentionParams p;
    int cta_per_head;  // ceil(queries / 256)
    int vec_out;       // output rows 16-byte addressable
};

__device__ __forceinline__ uint32_t tmem_lane_address(uint32_t base, int warp) {
    return base + (static_cast<uint32_t>((warp & 3) * 32) << 16);
}

// Descriptor start addresses count 16-byte units: one K=16 step of FP16 is 32 bytes (+2), the
// k1 half of a K row starts 64 bytes in (+4), and consecutive stages are one tile apart.
constexpr uint64_t kDescStep = 2, kDescHalf = 4, kDescStageK = kTileBytes / 16, kDescStageV = kVTileWords * 4 / 16;

// S(buffer) = q0.k1 + q1.k0 + q0.k0 over the 32 features (two K=16 steps each), then a commit
// to `bar`; k_desc addresses the stage's k16 tile. Warp-collective.
__device__ __forceinline__ void issue_scores(uint32_t tmem, uint64_t k_desc, int tile, int buffer, uint64_t *bar) {
    const uint32_t t = tmem + tile * kColTile;
    const uint32_t d = t + kColBuffer + buffer * kBufferColumns;
    const uint32_t a[4] = {t + kColQ0, t + kColQ0 + 8, t + kColQ1, t + kColQ1 + 8};
    const uint64_t bk[4] = {k_desc + kDescHalf, k_desc + kDescHalf + kDescStep, k_desc, k_desc + kDescStep};
    mma4_f16_ts_warp(d, a, bk, kIdescS, 1);
    mma2_f16_ts_commit_warp(d, t + kColQ0, t + kColQ0 + 8, k_desc, k_desc + kDescStep, kIdescS, bar);
}

// [Oa | Ob | sums] = p1.[v0 ; v1 ; 1] + p0.[v0 ; v1 ; 1] over the 64 keys (four K=16 steps
// each), then a commit to `bar`; v_desc addresses the stage's vt16 tile. Warp-collective.
__device__ __forceinline__ void issue_values(uint32_t tmem, uint64_t v_desc, int tile, int buffer, uint64_t *bar) {
    const uint32_t t = tmem + tile * kColTile;
    const uint32_t pbuf = t + kColBuffer + buffer * kBufferColumns;
    const uint64_t bv[4] = {v_desc, v_desc + kDescStep, v_desc + 2 * kDescStep, v_desc + 3 * kDescStep};
    const uint32_t a1[4] = {pbuf + 32, pbuf + 40, pbuf + 48, pbuf + 56};
    const uint32_t a0[4] = {pbuf, pbuf + 8, pbuf + 16, pbuf + 24};
    mma4_f16_ts_warp(t + kColO, a1, bv, kIdescPV, 1);
    mma4_f16_ts_commit_warp(t + kColO, a0, bv, kIdescPV, 0, bar);
}

// x' = x * scale split into (x0, x1): x0 exact in FP16, x1 = x' - x0 (rounded to FP16 on packing).
__device__ __forceinline__ void split_half(float x, float scale, float &x0, float &x1) {
    const float scaled = x * scale;
    x0 = round_tf32(scaled);  // 10 explicit mantissa bits, the FP16 precision
    x1 = scaled - x0;
}

// Folds the last finished key tile into the running output and row sum. In TMEM, Oa + Ob is the
// tile's P.V with V scaled by 2^c (c = the tile's V exponent) and the sum column its row sum of P.
// The running output is held as O * 2^o_exp, o_exp being the smallest V exponent folded so far:
// a tile with that exponent (the usual case, warp-uniform) costs one add and one FMA per column;
// a tile with another exponent moves whichever side has the larger one down, so no value is
// ever scaled up.
__device__ __forceinline__ void fold_output(float (&o)[32], float &row_sum, int &o_exp, uint32_t lane_base, float weight,
                                            int c) {
    if (o_exp == kNoExponent) o_exp = c;
    float out_weight = weight, tile_scale = 1.f;
    if (c > o_exp) {
        tile_scale = exp2_int(o_exp - c);
    } else if (c < o_exp) {
        out_weight = weight * exp2_int(c - o_exp);
        o_exp = c;
    }
    float oa[16], ob[16], sum;
    tmem_load16x2_1(lane_base + kColO, oa, lane_base + kColO + 32, ob, lane_base + kColSum, sum);
    row_sum = fmaf(row_sum, weight, sum);
    if (__all_sync(0xffffffffu, tile_scale == 1.f)) {  // uniform anyway; the loads inside are warp-collective
#pragma unroll
        for (int c = 0; c < 16; ++c) o[c] = fmaf(o[c], out_weight, oa[c] + ob[c]);
        tmem_load16x2(lane_base + kColO + 16, oa, lane_base + kColO + 48, ob);
#pragma unroll
        for (int c = 0; c < 16; ++c) o[16 + c] = fmaf(o[16 + c], out_weight, oa[c] + ob[c]);
    } else {
#pragma unroll
        for (int c = 0; c < 16; ++c) o[c] = fmaf(o[c], out_weight, (oa[c] + ob[c]) * tile_scale);
        tmem_load16x2(lane_base + kColO + 16, oa, lane_base + kColO + 48, ob);
#pragma unroll
        for (int c = 0; c < 16; ++c) o[16 + c] = fmaf(o[16 + c], out_weight, (oa[c] + ob[c]) * tile_scale);
    }
}

// P' = 2^14 exp(S - max) = exp2(S * slope + offset) of 64 scores, split into FP16 pairs: p0 =
// P' truncated to 11 significant bits (exact in FP16), p1 = FP16(P' - p0), stored to the P
// buffer (p0 pairs in columns 0-31, p1 pairs in 32-63) in chunks of 16 keys without waiting, so
// few values are live at a time. kPlain: every score is finite or -inf and the offset is finite,
// so exp2(-inf) = 0 covers the masked keys; otherwise -inf scores are zeroed explicitly (a row
// without any visible key yet has an infinite offset).
template <bool kPlain>
__device__ __forceinline__ void exp_split_store(const float (&sc)[64], float slope, float offset, uint32_t pbuf) {
#pragma unroll
    for (int chunk = 0; chunk < 4; ++chunk) {
        float p0[8], p1[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int c = 8 * chunk + i;
            float a = fast_exp2(fmaf(sc[2 * c], slope, offset));
            float b = fast_exp2(fmaf(sc[2 * c + 1], slope, offset));
            if (!kPlain) {
                a = sc[2 * c] == -INFINITY ? 0.f : a;
                b = sc[2 * c + 1] == -INFINITY ? 0.f : b;
            }
            const float a0 = __uint_as_float(__float_as_uint(a) & 0xFFFFE000u);
            const float b0 = __uint_as_float(__float_as_uint(b) & 0xFFFFE000u);
            p0[i] = __uint_as_float(pack_half2(a0, b0));
            p1[i] = __uint_as_float(pack_half2(a - a0, b - b0));
        }
        tmem_store8x2_async(pbuf + 8 * chunk, p0, pbuf + 32 + 8 * chunk, p1);
    }
}

__global__ void __launch_bounds__(kThreads, 1)
        flash_forward_kernel(const FlashArgs args, const __grid_constant__ CUtensorMap tmap_k,
                             const __grid_constant__ CUtensorMap tmap_v) {
    extern __shared__ uint8_t shared_raw[];
    SharedStorage &s = *reinterpret_cast<SharedStorage *>((reinterpret_cast<uintptr_t>(shared_raw) + 1023) & ~uintptr_t(1023));
    const AttentionParams &p = args.p;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    int block = blockIdx.x;
    const int cta_tile = block % args.cta_per_head;
    block /= args.cta_per_head;
    const int h = block % p.heads;
    const int b = block / p.heads;
    const int q0 = cta_tile * kCtaQueries;
    int first, last;
    key_window(q0, min(q0 + kCtaQueries, p.queries), p.keys, p.radius, first, last);
    const int tiles = last > first ? (last - first + kKeyTile - 1) / kKeyTile : 0;

    if (warp == 0) {
        tmem_alloc(&s.tmem_base, kTmemColumns);
        tmem_relinquish();
    }
    if (threadIdx.x == kProducerWarp * 32) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&s.kv_full[i], 1);
            mbar_init(&s.kv_ready[i], kSplitThreads);
            mbar_init(&s.kv_empty[i], 1);
        }
        for (int t = 0; t < kQTiles; ++t) {
            mbar_init(&s.s_full[t][0], 1);
            mbar_init(&s.s_full[t][1], 1);
            mbar_init(&s.p_full[t], kQTile);
            mbar_init(&s.pv_done[t], 1);
        }
        mbar_init(&s.q_ready, kQTile * kQTiles);
        mbar_init(&s.mma_done, 1);
        mbar_fence_init();
    }
    // Rows 64-79 of every V operand tile are FP16 ones, so P.V also yields the row sums of P.
    for (int i = threadIdx.x; i < kStages * 16 * 32; i += kThreads)
        s.vt16[i / (16 * 32)][2 * kD * 32 + i % (16 * 32)] = 0x3C003C00u;
    fence_proxy_async_shared();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s.tmem_base;

    if (warp == kProducerWarp) {
        // ---------------------------------------------------------------- TMA producer
        if (lane == 0) {
            int issued = 0;
            bool ok = true;
            for (int j = 0; j < tiles && ok; ++j) {
                const int stage = j % kStages, use = j / kStages;
                if (j >= kStages) ok = mbar_wait(&s.kv_empty[stage], (use - 1) & 1);
                if (!ok) break;
                RK_TRACE(j, 12);
                mbar_arrive_expect_tx(&s.kv_full[stage], 2 * kTileBytes);
                tma_load_4d(s.k_raw[stage], &tmap_k, &s.kv_full[stage], 0, first + j * kKeyTile, h, b);
                tma_load_4d(s.v_raw[stage], &tmap_v, &s.kv_full[stage], 0, first + j * kKeyTile, h, b);
                ++issued;
            }
            if (!ok) {
                // Do not leave copies in flight into shared memory of a finishing CTA.
                for (int j = max(0, issued - kStages); j < issued; ++j)
                    mbar_wait(&s.kv_full[j % kStages], (j / kStages) & 1);
            }
        }
    } else if (warp == kMmaWarp) {
        // ---------------------------------------------------------------- MMA issuer
        // S(t, 0) and S(t, 1) first; then for every key tile j, whichever Q tile's P is ready
        // first gets P(j).V and S(j + 2) (into the buffer P(j) occupied) issued first; the K/V
        // stage of tile j is released once both P.V products are issued. The whole warp runs
        // the loop (uniform control flow and descriptors); elected lanes issue the tcgen05 ops.
        if (tiles > 0) {
            const uint64_t k_desc0 = sw128_descriptor(smem_u32(s.k16[0]));
            const uint64_t v_desc0 = sw128_descriptor(smem_u32(s.vt16[0]));
            bool ok = mbar_wait_warp(&s.q_ready, 0);
            tc_fence_after();
            for (int j = 0; j < min(2, tiles) && ok; ++j) {
                ok = mbar_wait_warp(&s.kv_ready[j], 0);
                tc_fence_after();
                if (!ok) break;
#pragma unroll
                for (int t = 0; t < kQTiles; ++t) {
                    issue_scores(tmem, k_desc0 + kDescStageK * j, t, j, &s.s_full[t][j]);
                }
            }
            for (int j = 0; j < tiles && ok; ++j) {
                const int stage = j % kStages, buffer = j & 1;
                const bool more = j + 2 < tiles;
                const int next_stage = (j + 2) % kStages;
                bool next_ready = !more;
                bool served[kQTiles] = {false, false};
                const long long start_clock = clock64();
                int remaining = kQTiles;
                while (remaining > 0 && ok) {
#pragma unroll
                    for (int t = 0; t < kQTiles; ++t) {
                        if (!ok || served[t] || !mbar_test_wait_warp(&s.p_full[t], j & 1)) continue;
                        if (lane == 0) RK_TRACE(j, t);
                        tc_fence_after();
                        issue_values(tmem, v_desc0 + kDescStageV * stage, t, buffer, &s.pv_done[t]);
                        if (more) {
                            if (!next_ready) {
                                next_ready = mbar_wait_warp(&s.kv_ready[next_stage], ((j + 2) / kStages) & 1);
                                if (!next_ready) {
                                    ok = false;
                                    continue;
                                }
                                tc_fence_after();
                            }
                            issue_scores(tmem, k_desc0 + kDescStageK * next_stage, t, buffer, &s.s_full[t][buffer]);
                        }
                        served[t] = true;
                        --remaining;
                    }
                    if (remaining > 0 && ok && __any_sync(0xffffffffu, clock64() - start_clock > kWaitTimeoutCycles)) {
                        if (lane == 0) atomicOr(&g_device_status, kStatusWaitTimeout);
                        ok = false;
                    }
                }
                mma_commit_warp(&s.kv_empty[stage]);
            }
            // TMEM is released only after every issued MMA has completed.
            mma_commit_warp(&s.mma_done);
            mbar_wait_warp(&s.mma_done, 0);
        }
    } else if (warp >= kSplitWarp) {
        // ---------------------------------------------------------------- FP16 split
        // Split warp w owns key rows [32w, 32w + 32) of every tile; its ballot is their mask.
        // K: lane = one key row (8 raw 16-byte chunks in, 8 FP16 chunks [k0 | k1] out).
        // V: lane = (key group of 8 rows, chunk of 4 features): 8 raw chunks in, the 4 features'
        // 8-key FP16 chunks of v0^T and v1^T out.
        const int w = warp - kSplitWarp;
        const unsigned char *mask = p.mask + static_cast<long long>(b) * p.keys;
        const int row = 32 * w + lane;          // K row of this lane
        const int group = 4 * w + (lane >> 3);  // V key group (rows 8g..8g+7)
        const int fchunk = lane & 7;            // V logical feature chunk (features 4f..4f+3)
        for (int j = 0; j < tiles; ++j) {
            const int stage = j % kStages, use = j / kStages;
            // Both split warps pass the named barrier below before either may give up, so a
            // failed wait can never leave one of them blocked in bar.sync.
            const bool landed = __all_sync(0xffffffffu, mbar_wait(&s.kv_full[stage], use & 1));
            const int key = first + j * kKeyTile + row;
            const uint32_t bits = __ballot_sync(0xffffffffu, key < last && mask[key] != 0);
            const bool keep_row = (bits >> lane) & 1;
            const float4 *k4 = reinterpret_cast<const float4 *>(s.k_raw[stage]);
            const float4 *v4 = reinterpret_cast<const float4 *>(s.v_raw[stage]);
            float4 kx[8], vx[8];
            float kmax = 0.f, vmax = 0.f;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                kx[c] = k4[row * 8 + (c ^ (row & 7))];  // logical chunk c of the row
                if (!keep_row) kx[c] = make_float4(0.f, 0.f, 0.f, 0.f);
                kmax = fmaxf(kmax, fmaxf(fmaxf(fabsf(kx[c].x), fabsf(kx[c].y)), fmaxf(fabsf(kx[c].z), fabsf(kx[c].w))));
                const int vrow = 8 * group + c;
                vx[c] = v4[vrow * 8 + (fchunk ^ (vrow & 7))];
                if (!((bits >> (vrow & 31)) & 1)) vx[c] = make_float4(0.f, 0.f, 0.f, 0.f);
                vmax = fmaxf(vmax, fmaxf(fmaxf(fabsf(vx[c].x), fabsf(vx[c].y)), fmaxf(fabsf(vx[c].z), fabsf(vx[c].w))));
            }
#pragma unroll
            for (int offset = 16; offset; offset >>= 1) {
                kmax = fmaxf(kmax, __shfl_xor_sync(0xffffffffu, kmax, offset));
                vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, offset));
            }
            if (lane == 0) {
                s.split_max[w][0] = kmax;
                s.split_max[w][1] = vmax;
                s.split_ok[w] = landed;
                s.key_mask[stage][w] = bits;
            }
            asm volatile("bar.sync 1, 64;" ::: "memory");
            if (!(s.split_ok[0] && s.split_ok[1])) break;
            const int k_exponent = fp16_scale_exponent(fmaxf(s.split_max[0][0], s.split_max[1][0]));
            const int v_exponent = fp16_scale_exponent(fmaxf(s.split_max[0][1], s.split_max[1][1]));
            asm volatile("bar.sync 1, 64;" ::: "memory");  // split_max is rewritten for the next tile
            if (threadIdx.x == kSplitWarp * 32) {
                s.k_exponent[stage] = k_exponent;
                s.v_exponent[stage] = v_exponent;
            }
            const float k_scale = exp2_int(k_exponent), v_scale = exp2_int(v_exponent);
            // K row: features 8m..8m+7 -> k0 chunk m, k1 chunk 4 + m (16-byte chunks, swizzled by row % 8)
            uint4 *k16 = reinterpret_cast<uint4 *>(s.k16[stage]);
#pragma unroll
            for (int m = 0; m < 4; ++m) {
                const float x[8] = {kx[2 * m].x, kx[2 * m].y, kx[2 * m].z, kx[2 * m].w,
                                    kx[2 * m + 1].x, kx[2 * m + 1].y, kx[2 * m + 1].z, kx[2 * m + 1].w};
                float x0[8], x1[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) split_half(x[e], k_scale, x0[e], x1[e]);
                k16[row * 8 + (m ^ (row & 7))] = make_uint4(pack_half2(x0[0], x0[1]), pack_half2(x0[2], x0[3]),
                                                            pack_half2(x0[4], x0[5]), pack_half2(x0[6], x0[7]));
                k16[row * 8 + ((4 + m) ^ (row & 7))] = make_uint4(pack_half2(x1[0], x1[1]), pack_half2(x1[2], x1[3]),
                                                                  pack_half2(x1[4], x1[5]), pack_half2(x1[6], x1[7]));
            }
            // V^T rows f (v0) and 32 + f (v1), keys 8g..8g+7 = 16-byte chunk g (swizzled by f % 8)
            uint4 *vt16 = reinterpret_cast<uint4 *>(s.vt16[stage]);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int f = 4 * fchunk + e;
                float v0[8], v1[8];
#pragma unroll
                for (int r = 0; r < 8; ++r) {
                    const float value = e == 0 ? vx[r].x : e == 1 ? vx[r].y : e == 2 ? vx[r].z : vx[r].w;
                    split_half(value, v_scale, v0[r], v1[r]);
                }
                vt16[f * 8 + (group ^ (f & 7))] = make_uint4(pack_half2(v0[0], v0[1]), pack_half2(v0[2], v0[3]),
                                                             pack_half2(v0[4], v0[5]), pack_half2(v0[6], v0[7]));
                vt16[(32 + f) * 8 + (group ^ (f & 7))] = make_uint4(pack_half2(v1[0], v1[1]), pack_half2(v1[2], v1[3]),
                                                                    pack_half2(v1[4], v1[5]), pack_half2(v1[6], v1[7]));
            }
            fence_proxy_async_shared();
            if (lane == 0 && w == 0) RK_TRACE(j, 3);
            mbar_arrive(&s.kv_ready[stage]);
        }
    } else {
        // ---------------------------------------------------------------- softmax / epilogue
        const int tile = warp >> 2;  // 0 = A, 1 = B
        const int row_in_tile = threadIdx.x & (kQTile - 1);
        const int query = q0 + tile * kQTile + row_in_tile;
        const bool row_valid = query < p.queries;
        const uint32_t lane_base = tmem_lane_address(tmem, warp) + tile * kColTile;
        const bool tracer = row_in_tile == 0;

        int q_exponent;
        {  // Q row -> scaled by 1/sqrt(D) and 2^q_exponent, split into FP16 q0/q1 pairs in TMEM
            float x[32];
            const float4 *q4 = reinterpret_cast<const float4 *>(p.q.row(b, h, row_valid ? query : 0));
            float qmax = 0.f;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const float4 v = row_valid ? __ldg(q4 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
                x[4 * c] = v.x * p.scale;
                x[4 * c + 1] = v.y * p.scale;
                x[4 * c + 2] = v.z * p.scale;
                x[4 * c + 3] = v.w * p.scale;
#pragma unroll
                for (int e = 0; e < 4; ++e) qmax = fmaxf(qmax, fabsf(x[4 * c + e]));
            }
            q_exponent = fp16_scale_exponent(qmax);
            const float q_scale = exp2_int(q_exponent);
            float packed0[16], packed1[16];
#pragma unroll
            for (int c = 0; c < 16; ++c) {
                float a0, a1, b0, b1;
                split_half(x[2 * c], q_scale, a0, a1);
                split_half(x[2 * c + 1], q_scale, b0, b1);
                packed0[c] = __uint_as_float(pack_half2(a0, b0));
                packed1[c] = __uint_as_float(pack_half2(a1, b1));
            }
            tmem_store16x2(lane_base + kColQ0, packed0, lane_base + kColQ1, packed1);
            tc_fence_before();
            mbar_arrive(&s.q_ready);
        }

        float row_max = -INFINITY, row_sum = 0.f;  // row_sum carries the 2^14 of P
        float o[32];                               // running output, scaled by 2^o_exp
#pragma unroll
        for (int c = 0; c < 32; ++c) o[c] = 0.f;
        int o_exp = kNoExponent;
        float pending_weight = 0.f;  // exp(m_(j-2) - m_(j-1)), applied when tile j-1 is folded
        int pending_exponent = 0;    // c_(j-1): the V exponent of tile j-1
        bool ok = true;
        for (int j = 0; j < tiles && ok; ++j) {
            const int stage = j % kStages, use = j / kStages, buffer = j & 1;
            const uint32_t pbuf = lane_base + kColBuffer + buffer * kBufferColumns;
            ok = __all_sync(0xffffffffu, mbar_wait(&s.s_full[tile][buffer], (j >> 1) & 1) &&
                                                 mbar_wait(&s.kv_ready[stage], use & 1));
            if (!ok) break;
            if (tracer) RK_TRACE(j, 4 + 4 * tile);
            RK_WARP_TRACE(j, 0);
            tc_fence_after();
            float sc[64];
            tmem_load64(pbuf, sc);
            // Visible keys of this row in the tile: key mask x radius window x valid row.
            const int k0 = first + j * kKeyTile;
            uint64_t active = row_valid ? (static_cast<uint64_t>(s.key_mask[stage][0]) |
                                           (static_cast<uint64_t>(s.key_mask[stage][1]) << 32))
                                        : 0ull;
            if (p.radius >= 0) {
                const int lo_col = max(0, query - p.radius - k0), hi_col = min(kKeyTile - 1, query + p.radius - k0);
                active &= lo_col > hi_col ? 0ull : ((~0ull) >> (63 - (hi_col - lo_col))) << lo_col;
            }
            const float s_scale = exp2_int(-(q_exponent + s.k_exponent[stage]));  // TMEM S -> scaled score
            const int v_exponent = s.v_exponent[stage];
            // Row max (four independent three-input max chains).
            if (active != ~0ull) {
#pragma unroll
                for (int c = 0; c < 64; ++c) sc[c] = (active >> c) & 1 ? sc[c] : -INFINITY;
            }
            float partial_max[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
            for (int c = 0; c < 64; c += 2) partial_max[(c >> 1) & 3] = max3(partial_max[(c >> 1) & 3], sc[c], sc[c + 1]);
            const float raw_max = max3(partial_max[0], partial_max[1], fmaxf(partial_max[2], partial_max[3]));
            const float tile_max = raw_max == -INFINITY ? -INFINITY : raw_max * s_scale;
            if (tracer) RK_TRACE(j, 5 + 4 * tile);
            RK_WARP_TRACE(j, 1);
            const float next = fmaxf(row_max, tile_max);
            const float old_weight = isfinite(row_max) ? fast_exp2((row_max - next) * kLog2e) : 0.f;
            const float slope = s_scale * kLog2e;
            const float offset = fmaf(-next, kLog2e, 14.f);  // P' = 2^14 exp(S - max) = exp2(S * slope + offset)
            // P(j) may be written before Ot(j - 1) is folded: only the p_full arrival below lets
            // the MMA warp start P(j).V, which overwrites Ot. The TMEM stores inside are
            // warp-collective, so the branch is taken by the whole warp (the explicit path is
            // exact for finite rows too).
            if (__all_sync(0xffffffffu, isfinite(offset) && slope > 0.f))
                exp_split_store<true>(sc, slope, offset, pbuf);
            else
                exp_split_store<false>(sc, slope, offset, pbuf);
            RK_WARP_TRACE(j, 2);
            if (j > 0) {  // fold tile j-1 before P(j).V overwrites its Ot
                ok = __all_sync(0xffffffffu, mbar_wait(&s.pv_done[tile], (j - 1) & 1));
                if (!ok) {
                    tmem_wait_store();  // no store may be in flight when TMEM is released
                    break;
                }
                tc_fence_after();
                fold_output(o, row_sum, o_exp, lane_base, pending_weight, pending_exponent);
            }
            RK_WARP_TRACE(j, 3);
            tmem_wait_store();
            RK_WARP_TRACE(j, 4);
            tc_fence_before();
            if (tracer) RK_TRACE(j, 6 + 4 * tile);
            mbar_arrive(&s.p_full[tile]);
            row_max = next;
            pending_weight = old_weight;
            pending_exponent = v_exponent;
        }

        // Epilogue (AttentionFlash32.h:157-169): O / total; fully masked rows give 0 and {-inf, 0}.
        if (tiles > 0 && ok) {
            ok = __all_sync(0xffffffffu, mbar_wait(&s.pv_done[tile], (tiles - 1) & 1));
            tc_fence_after();
            if (ok) fold_output(o, row_sum, o_exp, lane_base, pending_weight, pending_exponent);
        }
        if (row_valid) {
            const float total = ok ? row_sum : NAN;
            float *out = p.o.row(b, h, query);
            const float out_scale = exp2_int(-o_exp) / total;
#pragma unroll
            for (int c = 0; c < 32; ++c) o[c] = total > 0.f ? o[c] * out_scale : isnan(total) ? NAN : 0.f;
            if (args.vec_out) {
#pragma unroll
                for (int c = 0; c < 8; ++c)
                    reinterpret_cast<float4 *>(out)[c] = make_float4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
            } else {
#pragma unroll
                for (int c = 0; c < 32; ++c) out[c] = o[c];
            }
            const long long row = (static_cast<long long>(b) * p.heads + h) * p.queries + query;
            p.lse[row * 2] = total > 0.f ? row_max : isnan(total) ? NAN : -INFINITY;
            p.lse[row * 2 + 1] = total > 0.f ? total * (1.f / kPScale) : isnan(total) ? NAN : 0.f;
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemColumns);
    }
}

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

// [batch][heads][tokens][32] FP32 with the given element strides; box = 32 features x rows tokens.
bool make_tensor_map(CUtensorMap *map, const Tensor &t, int batch, int heads, int tokens, int rows) {
    auto encode = encode_function();
    if (encode == nullptr) return false;
    const cuuint64_t dims[4] = {kD, static_cast<cuuint64_t>(tokens), static_cast<cuuint64_t>(heads), static_cast<cuuint64_t>(batch)};
    const cuuint64_t strides[3] = {static_cast<cuuint64_t>(t.st) * 4, static_cast<cuuint64_t>(t.sh) * 4,
                                   static_cast<cuuint64_t>(t.sb) * 4};
    const cuuint32_t box[4] = {kD, static_cast<cuuint32_t>(rows), 1, 1};
    const cuuint32_t element_strides[4] = {1, 1, 1, 1};
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float *>(t.data), dims, strides, box, element_strides,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool positive_tma_strides(const Tensor &t) {
    const long long limit = 1ll << 38;  // strides below 2^40 bytes
    return t.st > 0 && t.sh > 0 && t.sb > 0 && t.st % 4 == 0 && t.sh % 4 == 0 && t.sb % 4 == 0 && t.st < limit &&
           t.sh < limit && t.sb < limit && (reinterpret_cast<uintptr_t>(t.data) & 15u) == 0;
}

constexpr int kSharedBytes = static_cast<int>(sizeof(SharedStorage)) + 1024;
static_assert(sizeof(SharedStorage::k16[0]) == 64 * 128 && sizeof(SharedStorage::vt16[0]) == kVRows * 128,
              "FP16 operand tiles are rows of 128 bytes");
static_assert(sizeof(SharedStorage::vt16[0]) % 1024 == 0, "V operand tiles stay 1024-byte aligned");
static_assert(kColSum + 16 <= kColTile, "Q tile TMEM columns");
static_assert(kSharedBytes <= 227 * 1024, "shared memory budget");

}  // namespace

bool flash_supported(const AttentionParams &p) {
    return p.vec4 && positive_tma_strides(p.k) && positive_tma_strides(p.v) && (p.q.st % 4 == 0) &&
           (reinterpret_cast<uintptr_t>(p.q.data) & 15u) == 0;
}

int launch_flash_forward(const AttentionParams &p, cudaStream_t stream) {
    CUtensorMap tmap_k, tmap_v;
    if (!make_tensor_map(&tmap_k, p.k, p.batch, p.heads, p.keys, kKeyTile) ||
        !make_tensor_map(&tmap_v, p.v, p.batch, p.heads, p.keys, kKeyTile))
        return kNotEligible;
    cudaError_t status = prepare_kernel<flash_forward_kernel>(kSharedBytes);
    if (status != cudaSuccess) return status;
    FlashArgs args{};
    args.p = p;
    args.cta_per_head = (p.queries + kCtaQueries - 1) / kCtaQueries;
    args.vec_out = (reinterpret_cast<uintptr_t>(p.o.data) & 15u) == 0 && p.o.sb % 4 == 0 && p.o.sh % 4 == 0 && p.o.st % 4 == 0;
    const unsigned blocks = static_cast<unsigned>(args.cta_per_head) * static_cast<unsigned>(p.heads) * static_cast<unsigned>(p.batch);
    flash_forward_kernel<<<blocks, kThreads, kSharedBytes, stream>>>(args, tmap_k, tmap_v);
    return cudaGetLastError();
}

unsigned int read_device_status(bool clear) {
    unsigned int value = 0;
    if (cudaMemcpyFromSymbol(&value, g_device_status, sizeof(value)) != cudaSuccess) return ~0u;
    if (clear && value != 0) {
        const unsigned int zero = 0;
        cudaMemcpyToSymbol(g_device_status, &zero, sizeof(zero));
    }
    return value;
}

const char *kernel_name() { return "tcgen05-f16x2-flash-d32"; }

#ifdef RK_TC_TRACE
extern "C" __attribute__((visibility("default"))) int rocmkernels_attention_trace(long long *out, int capacity) {
    const int count = kTraceTiles * kTraceEvents;
    if (capacity < count) return -1;
    if (cudaMemcpyFromSymbol(out, g_trace, sizeof(long long) * count) != cudaSuccess) return -2;
    if (capacity >= count + 64 && cudaMemcpyFromSymbol(out + count, g_warp_trace, sizeof(long long) * 64) != cudaSuccess) return -3;
    return count;
}
#endif

const char *build_info() {
    return "sm_100a; tcgen05-f16x2-flash-d32 forward (TMA + TMEM, split FP16 operands, double-buffered S, tensor-core row sums); "
           "simt-fp32 d32/d64 forward+backward";
}

}  // namespace tc
}  // namespace rk
