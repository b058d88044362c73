// Tensor-core flash forward for head width 32 on sm_100a: tcgen05.mma (kind::tf32) with TMEM
// accumulators, TMA-staged K/V tiles and 3xTF32 error compensation.
//
// Replaces the reference's flash forward (attention_query_flash_body, AttentionFlash32.h:23-170):
// same results (O = softmax(scale * Q K^T, masked) V, lse = {row max, exp sum}), same masking
// and radius rules, same fully-masked / NaN conventions; different machine.
//
// CTA = 256 queries as two 128-row Q tiles ("A" and "B") that share every K/V tile.
//   warps 0-3   softmax + epilogue of Q tile A (thread = query row = TMEM lane)
//   warps 4-7   softmax + epilogue of Q tile B
//   warp  8     TMA producer: K and V tiles of 64 keys x 32 features, 128B swizzle
//   warp  9     MMA issuer (one thread)
//   warps 10-11 split each K tile into TF32 hi/lo rows and each V tile into transposed hi/lo
//               rows, zero masked key rows, publish the tile's key mask
//
// 3xTF32 with operands stacked along N. A tcgen05.mma kind::tf32 (M=128, K=8) costs about 46
// cycles for any N <= 64 and reaches full rate only at N >= 128, so the hi/lo products are
// packed into as few, as wide, instructions as possible:
//   S  : [X | Y] = Qhi . [Khi ; Klo]^T  (N=128), then X += Qlo . Khi^T (N=64);  S = X + Y
//   PV : [Oa | Ob] = Phi . [Vhi ; Vlo] + Plo . [Vhi ; Vlo]  (N=64 each);          Ot = Oa + Ob
// Q (hi, lo) and P (hi over X, lo over Y) are the A operands in TMEM; K and V^T are the B
// operands in shared memory, 128B-swizzled K-major (keys resp. features as rows). V is used
// transposed because the split warps write it so while splitting.
// Each key tile's Ot is folded into the running output in FP32 registers by the softmax
// threads (O = O * exp(m_old - m_new) + Ot, with the running max and sum; online softmax as in
// AttentionFlash32.h:96-112). Folding in registers keeps the cross-tile sum in round-to-nearest
// FP32; accumulating all tiles in one tensor-core accumulator lost about 1e-6 per tile.
//
// TMEM (512 columns, one CTA per SM), Q tile t uses [256t, 256t + 256):
//   Qhi 0-31 | Qlo 32-63 | X (S part, then Phi) 64-127 | Y (S part, then Plo) 128-191 | Oa 192-223 | Ob 224-255
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
#define RK_TRACE(tile_index, event)                                                              \
    do {                                                                                        \
        if (blockIdx.x == 0 && (tile_index) < kTraceTiles) g_trace[(tile_index)][(event)] = clock64(); \
    } while (0)
#else
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
constexpr uint32_t kTmemColumns = 512;
constexpr uint32_t kColQhi = 0, kColQlo = 32, kColX = 64, kColY = 128, kColO = 192, kColTile = 256;
constexpr uint32_t kIdescS2 = tf32_instr_desc(128, 2 * kKeyTile, false);  // Qhi . [Khi ; Klo]
constexpr uint32_t kIdescS1 = tf32_instr_desc(128, kKeyTile, false);      // Qlo . Khi
constexpr uint32_t kIdescPV = tf32_instr_desc(128, 2 * kD, false);        // P . [Vhi ; Vlo]

struct alignas(1024) SharedStorage {
    float k[kStages][2 * kTileFloats];  // rows 0-63: raw K as TMA lands it, rewritten as Khi; rows 64-127: Klo
    float v[kStages][kTileFloats];      // raw V as TMA lands it
    float vt[kStages][2 * kTileFloats]; // [Vhi^T ; Vlo^T]: 64 rows (hi features 0-31, lo features 0-31) x 64 keys,
                                        // as two 8 KB atom columns of 32 keys, K-major 128B swizzle
    uint32_t key_mask[kStages][2];     // bit c: key k0 + c visible
    uint64_t kv_full[kStages];         // TMA bytes landed
    uint64_t kv_ready[kStages];        // split done (64 arrivals)
    uint64_t kv_empty[kStages];        // MMAs reading the stage finished (commit)
    uint64_t s_full[kQTiles];          // S of the current tile is in TMEM (commit)
    uint64_t p_full[kQTiles];          // P of the current tile is in TMEM (128 arrivals)
    uint64_t pv_done[kQTiles];         // O += P V finished (commit)
    uint64_t q_ready;                  // Q hi/lo of both tiles in TMEM (256 arrivals)
    uint64_t mma_done;                 // every MMA of the CTA finished (commit)
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

__device__ void issue_scores(SharedStorage &s, uint32_t tmem, int tile, int stage) {
    const uint32_t t = tmem + tile * kColTile;
    const uint32_t k = smem_u32(s.k[stage]);
#pragma unroll
    for (int kk = 0; kk < kD / 8; ++kk)
        mma_tf32_ts(t + kColX, t + kColQhi + 8 * kk, sw128_descriptor(k + 32 * kk), kIdescS2, kk > 0);
#pragma unroll
    for (int kk = 0; kk < kD / 8; ++kk)
        mma_tf32_ts(t + kColX, t + kColQlo + 8 * kk, sw128_descriptor(k + 32 * kk), kIdescS1, 1);
}

__device__ void issue_values(SharedStorage &s, uint32_t tmem, int tile, int stage) {
    const uint32_t t = tmem + tile * kColTile;
    const uint32_t v = smem_u32(s.vt[stage]);
    // k-step kk covers keys 8kk..8kk+7: atom column kk/4 (8 KB apart), 32 B into its rows.
#pragma unroll
    for (int kk = 0; kk < kKeyTile / 8; ++kk)
        mma_tf32_ts(t + kColO, t + kColX + 8 * kk, sw128_descriptor(v + 8192 * (kk / 4) + 32 * (kk % 4)), kIdescPV, kk > 0);
#pragma unroll
    for (int kk = 0; kk < kKeyTile / 8; ++kk)
        mma_tf32_ts(t + kColO, t + kColY + 8 * kk, sw128_descriptor(v + 8192 * (kk / 4) + 32 * (kk % 4)), kIdescPV, 1);
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
            mbar_init(&s.s_full[t], 1);
            mbar_init(&s.p_full[t], kQTile);
            mbar_init(&s.pv_done[t], 1);
        }
        mbar_init(&s.q_ready, kQTile * kQTiles);
        mbar_init(&s.mma_done, 1);
        mbar_fence_init();
    }
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
                tma_load_4d(s.k[stage], &tmap_k, &s.kv_full[stage], 0, first + j * kKeyTile, h, b);
                tma_load_4d(s.v[stage], &tmap_v, &s.kv_full[stage], 0, first + j * kKeyTile, h, b);
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
        // For every key tile, whichever Q tile's P is ready first gets its P.V (and the next S)
        // issued first; the K/V stage is released once both P.V products are issued.
        if (lane == 0 && tiles > 0) {
            bool ok = mbar_wait(&s.q_ready, 0) && mbar_wait(&s.kv_ready[0], 0);
            tc_fence_after();
            if (ok) {
                issue_scores(s, tmem, 0, 0);
                mma_commit(&s.s_full[0]);
                issue_scores(s, tmem, 1, 0);
                mma_commit(&s.s_full[1]);
            }
            for (int j = 0; j < tiles && ok; ++j) {
                const int stage = j % kStages;
                const bool more = j + 1 < tiles;
                const int next_stage = (j + 1) % kStages;
                bool next_ready = !more;
                bool served[kQTiles] = {false, false};
                const long long start_clock = clock64();
                int remaining = kQTiles;
                while (remaining > 0) {
                    for (int t = 0; t < kQTiles; ++t) {
                        if (served[t] || !mbar_try_wait(&s.p_full[t], j & 1)) continue;
                        RK_TRACE(j, t);
                        tc_fence_after();
                        issue_values(s, tmem, t, stage);
                        mma_commit(&s.pv_done[t]);
                        if (more) {
                            if (!next_ready) {
                                next_ready = mbar_wait(&s.kv_ready[next_stage], ((j + 1) / kStages) & 1);
                                if (!next_ready) break;
                                tc_fence_after();
                            }
                            issue_scores(s, tmem, t, next_stage);
                            mma_commit(&s.s_full[t]);
                        }
                        served[t] = true;
                        --remaining;
                    }
                    if (more && !next_ready && remaining < kQTiles) { ok = false; break; }
                    if (remaining > 0 && clock64() - start_clock > kWaitTimeoutCycles) {
                        atomicOr(&g_device_status, kStatusWaitTimeout);
                        ok = false;
                        break;
                    }
                }
                mma_commit(&s.kv_empty[stage]);
            }
            // TMEM is released only after every issued MMA has completed.
            mma_commit(&s.mma_done);
            mbar_wait(&s.mma_done, 0);
        }
    } else if (warp >= kSplitWarp) {
        // ---------------------------------------------------------------- hi/lo split
        // Split warp w owns key rows [32w, 32w + 32) of every tile: its ballot is their mask.
        // K: each lane rewrites 8 of the warp's 256 swizzled 16-byte chunks in place (hi) and
        // into k_lo. V: each lane takes 2 (4-key group, 4-feature chunk) items, reads the 4 rows
        // and writes 4 features x 4 keys of V^T hi and lo as 16-byte stores.
        const int w = warp - kSplitWarp;
        const unsigned char *mask = p.mask + static_cast<long long>(b) * p.keys;
        for (int j = 0; j < tiles; ++j) {
            const int stage = j % kStages, use = j / kStages;
            if (!__all_sync(0xffffffffu, mbar_wait(&s.kv_full[stage], use & 1))) break;
            const int key = first + j * kKeyTile + 32 * w + lane;
            const uint32_t bits = __ballot_sync(0xffffffffu, key < last && mask[key] != 0);
            if (lane == 0) s.key_mask[stage][w] = bits;
            float4 *k4 = reinterpret_cast<float4 *>(s.k[stage]);
            float4 *klo4 = k4 + kTileFloats / 4;
#pragma unroll 4
            for (int it = 0; it < 8; ++it) {
                const int chunk = 256 * w + 32 * it + lane;
                const bool keep = (bits >> ((chunk >> 3) & 31)) & 1;
                const float4 x = k4[chunk];
                float4 hi, lo;
                split_tf32(keep ? x.x : 0.f, hi.x, lo.x);
                split_tf32(keep ? x.y : 0.f, hi.y, lo.y);
                split_tf32(keep ? x.z : 0.f, hi.z, lo.z);
                split_tf32(keep ? x.w : 0.f, hi.w, lo.w);
                k4[chunk] = hi;
                klo4[chunk] = lo;
            }
            const float4 *v4 = reinterpret_cast<const float4 *>(s.v[stage]);
            float4 *vt = reinterpret_cast<float4 *>(s.vt[stage]);
#pragma unroll
            for (int it = 0; it < 2; ++it) {
                const int item = 32 * it + lane;        // 64 items per warp: 8 key groups x 8 chunks
                const int group = 8 * w + (item >> 3);  // 4-key group 0..15 (rows 4g..4g+3)
                const int chunk = item & 7;             // logical 4-feature chunk
                float rows[4][4];
#pragma unroll
                for (int rr = 0; rr < 4; ++rr) {
                    const int row = 4 * group + rr;
                    const bool keep = (bits >> (row & 31)) & 1;
                    const float4 y = v4[row * 8 + (chunk ^ (row & 7))];
                    rows[rr][0] = keep ? y.x : 0.f;
                    rows[rr][1] = keep ? y.y : 0.f;
                    rows[rr][2] = keep ? y.z : 0.f;
                    rows[rr][3] = keep ? y.w : 0.f;
                }
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int f = 4 * chunk + e;
                    // keys 4g..4g+3 of rows f (hi) and 32 + f (lo): atom column g/8 (512 chunks),
                    // 16-byte chunk (g % 8) ^ (row % 8) of the 128-byte row.
                    const int index = (group >> 3) * 512 + f * 8 + ((group & 7) ^ (f & 7));
                    float4 hi, lo;
                    split_tf32(rows[0][e], hi.x, lo.x);
                    split_tf32(rows[1][e], hi.y, lo.y);
                    split_tf32(rows[2][e], hi.z, lo.z);
                    split_tf32(rows[3][e], hi.w, lo.w);
                    vt[index] = hi;
                    vt[index + 32 * 8] = lo;
                }
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

        {  // Q row -> scaled, split into TF32 hi/lo, stored as the A operand in TMEM
            float hi[32], lo[32];
            const float4 *q4 = reinterpret_cast<const float4 *>(p.q.row(b, h, row_valid ? query : 0));
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                float4 x = row_valid ? __ldg(q4 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
                split_tf32(x.x * p.scale, hi[4 * c], lo[4 * c]);
                split_tf32(x.y * p.scale, hi[4 * c + 1], lo[4 * c + 1]);
                split_tf32(x.z * p.scale, hi[4 * c + 2], lo[4 * c + 2]);
                split_tf32(x.w * p.scale, hi[4 * c + 3], lo[4 * c + 3]);
            }
            tmem_store32(lane_base + kColQhi, hi);
            tmem_store32(lane_base + kColQlo, lo);
            tc_fence_before();
            mbar_arrive(&s.q_ready);
        }

        float row_max = -INFINITY, row_sum = 0.f;
        float o[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) o[c] = 0.f;
        float pending_weight = 0.f;  // exp(m_(j-2) - m_(j-1)), applied when tile j-1's Ot is folded
        bool ok = true;
        for (int j = 0; j < tiles && ok; ++j) {
            const int stage = j % kStages, use = j / kStages;
            ok = __all_sync(0xffffffffu, mbar_wait(&s.s_full[tile], j & 1) && mbar_wait(&s.kv_ready[stage], use & 1));
            if (!ok) break;
            const bool tracer = (threadIdx.x & (kQTile - 1)) == 0;
            if (tracer) RK_TRACE(j, 4 + 4 * tile);
            if (j > 0) {
                // S_j was issued after P_(j-1).V, so Ot of tile j-1 is complete: fold it first.
                ok = __all_sync(0xffffffffu, mbar_wait(&s.pv_done[tile], (j - 1) & 1));
                if (!ok) break;
                tc_fence_after();
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    float oa[16], ob[16];
                    tmem_load16x2(lane_base + kColO + 16 * half, oa, lane_base + kColO + 32 + 16 * half, ob);
#pragma unroll
                    for (int c = 0; c < 16; ++c) o[16 * half + c] = fmaf(o[16 * half + c], pending_weight, oa[c] + ob[c]);
                }
            } else {
                tc_fence_after();
            }
            // Visible keys of this row in the tile: key mask x radius window x valid row.
            const int k0 = first + j * kKeyTile;
            uint64_t active = row_valid ? (static_cast<uint64_t>(s.key_mask[stage][0]) |
                                           (static_cast<uint64_t>(s.key_mask[stage][1]) << 32))
                                        : 0ull;
            if (p.radius >= 0) {
                const int lo_col = max(0, query - p.radius - k0), hi_col = min(kKeyTile - 1, query + p.radius - k0);
                active &= lo_col > hi_col ? 0ull : ((~0ull) >> (63 - (hi_col - lo_col))) << lo_col;
            }
            const bool all_active = active == ~0ull;
            // S = X + Y, masked, and its row max (4 independent max chains).
            float sc[64];
            float partial_max[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
            for (int quarter = 0; quarter < 4; ++quarter) {
                float x[16], y[16];
                tmem_load16x2(lane_base + kColX + 16 * quarter, x, lane_base + kColY + 16 * quarter, y);
#pragma unroll
                for (int c = 0; c < 16; ++c) {
                    const int column = 16 * quarter + c;
                    const float score = x[c] + y[c];
                    sc[column] = all_active || ((active >> column) & 1) ? score : -INFINITY;
                    partial_max[c & 3] = fmaxf(partial_max[c & 3], sc[column]);
                }
            }
            const float tile_max = fmaxf(fmaxf(partial_max[0], partial_max[1]), fmaxf(partial_max[2], partial_max[3]));
            if (tracer) RK_TRACE(j, 5 + 4 * tile);
            const float next = fmaxf(row_max, tile_max);
            const float old_weight = isfinite(row_max) ? fast_exp2((row_max - next) * kLog2e) : 0.f;
            const float offset = -next * kLog2e;
            // P = exp(S - max) (exp2(-inf) = 0 covers masked scores while the offset is finite)
            float partial_sum[4] = {0.f, 0.f, 0.f, 0.f};
            if (isfinite(offset)) {
#pragma unroll
                for (int c = 0; c < 64; ++c) {
                    sc[c] = fast_exp2(fmaf(sc[c], kLog2e, offset));
                    partial_sum[c & 3] += sc[c];
                }
            } else {
#pragma unroll
                for (int c = 0; c < 64; ++c) {
                    sc[c] = sc[c] == -INFINITY ? 0.f : fast_exp2(fmaf(sc[c], kLog2e, offset));
                    partial_sum[c & 3] += sc[c];
                }
            }
            const float tile_sum = (partial_sum[0] + partial_sum[1]) + (partial_sum[2] + partial_sum[3]);
            // TF32 split: Phi over X, Plo over Y.
#pragma unroll
            for (int quarter = 0; quarter < 4; ++quarter) {
                float lo[16];
#pragma unroll
                for (int c = 0; c < 16; ++c) {
                    float hi;
                    split_tf32(sc[16 * quarter + c], hi, lo[c]);
                    sc[16 * quarter + c] = hi;
                }
                tmem_store16x2(lane_base + kColX + 16 * quarter, sc + 16 * quarter, lane_base + kColY + 16 * quarter, lo);
            }
            tc_fence_before();
            if (tracer) RK_TRACE(j, 6 + 4 * tile);
            mbar_arrive(&s.p_full[tile]);
            row_sum = row_sum * old_weight + tile_sum;
            row_max = next;
            pending_weight = old_weight;
        }

        // Epilogue (AttentionFlash32.h:157-169): O / total; fully masked rows give 0 and {-inf, 0}.
        if (tiles > 0 && ok) {
            ok = __all_sync(0xffffffffu, mbar_wait(&s.pv_done[tile], (tiles - 1) & 1));
            tc_fence_after();
            if (ok) {
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    float oa[16], ob[16];
                    tmem_load16x2(lane_base + kColO + 16 * half, oa, lane_base + kColO + 32 + 16 * half, ob);
#pragma unroll
                    for (int c = 0; c < 16; ++c) o[16 * half + c] = fmaf(o[16 * half + c], pending_weight, oa[c] + ob[c]);
                }
            }
        }
        if (row_valid) {
            const float total = ok ? row_sum : NAN;
            float *out = p.o.row(b, h, query);
#pragma unroll
            for (int c = 0; c < 32; ++c) o[c] = total > 0.f ? o[c] / total : isnan(total) ? NAN : 0.f;
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
            p.lse[row * 2 + 1] = total > 0.f ? total : isnan(total) ? NAN : 0.f;
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

const char *kernel_name() { return "tcgen05-3xtf32-flash-d32"; }

#ifdef RK_TC_TRACE
extern "C" __attribute__((visibility("default"))) int rocmkernels_attention_trace(long long *out, int capacity) {
    const int count = kTraceTiles * kTraceEvents;
    if (capacity < count) return -1;
    return cudaMemcpyFromSymbol(out, g_trace, sizeof(long long) * count) == cudaSuccess ? count : -2;
}
#endif

const char *build_info() {
    return "sm_100a; tcgen05-3xtf32-flash-d32 forward (TMA + TMEM, N-stacked hi/lo operands); simt-fp32 d32/d64 forward+backward";
}

}  // namespace tc
}  // namespace rk
