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
// Prepared operands (the d = 32 split-FP32 forward given a caller workspace, where it pays):
// prepare_kv_kernel first converts every 64-key tile of every head once, into the byte image of
// that shared-memory stage plus a 16-byte header (mask bits, exponents); the forward then runs
//   warps 0-7   softmax + epilogue of Q tiles A and B (as above)
//   warp  8     producer: three bulk copies per key tile (K rows, V^T rows, header)
//   warps 9-10  MMA issuers, one per Q tile, each waiting (suspended) for its own P tiles
// with no split warps: the conversion is not repeated by each of a head's query blocks. The V rows
// of an image are [v1^T ; v0^T] (the ones follow in shared memory), so P.V accumulates
// Ot = p1.v0 + p0.v1 + p0.v0 in one 32-column accumulator (N = 48, 32, 48; the p1.v1 term, ~2^-22
// of the output, is left out) and the softmax threads fold one 33-column TMEM load per tile.
// TMEM per Q tile: q0 0-15 | q1 16-31 | S/P buffers 32-95, 96-159 | Ot 160-191 | row sums 192-207.
//
// Split FP16 operands. Every FP32 operand x is scaled by a power of two 2^e (Q: per row; K, V:
// per tile; P: 2^14) so that its largest magnitude lies in [2^14, 2^15), then split
// x' = x0 + x1: for Q, K and V x0 = FP16(x') (cvt.rn: 11 significant bits) and x1 = FP16(x' - x0),
// the residual taken from x0 widened back (tc_operands.cuh, split_pack2); for P x0 = P' with its
// low 13 mantissa bits cleared (also exact in FP16) and x1 = FP16(P' - x0). Products keep ~22 bits:
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
//
// FP16 storage (the generic forward's DType::Float16, attention_generic_query_half,
// AttentionGeneric.hip:141-237; head width 16, 32 or 64). The same pipeline with one FP16 term
// per operand and no scale exponents: the inputs already are FP16, so S = q.k is one product per
// K=16 step, read by the MMAs straight from the TMA tile of K (64 keys x 64 FP16, 128B swizzle;
// the features past D are the TMA's zero fill), and P is rounded to FP16 once for P.V (as the
// reference rounds it before its v_dot2 P.V) while the row sum adds the unrounded FP32 values
// (as the reference's total does). One Q tile per CTA; the split warps only transpose V and
// publish the key mask. The 1/sqrt(D) scale multiplies the FP32 scores, as in the reference.
// TMEM (256 columns): q 0..D/2-1 | S/P buffers 32-95, 96-159 (P in the first 32 columns) |
// O 160..160+D-1.
#include "attention_tc.cuh"

#include <cudaTypedefs.h>

#include <mutex>
#include <type_traits>

#include "rotary.cuh"
#include "tc_operands.cuh"


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
// per softmax warp, tile 30 of CTA 0: events 0 s_full seen, 1 max done, 2 exp and P stores issued,
// 3 fold done, 4 P stores complete
__device__ long long g_warp_trace[8][8];
#define RK_WARP_TRACE(tile_index, event)                                                                          \
    do {                                                                                                         \
        if (blockIdx.x == 0 && (tile_index) == 30 && (threadIdx.x & 31) == 0) g_warp_trace[threadIdx.x >> 5][(event)] = clock64(); \
    } while (0)
// per CTA (thread 0): events 0 entry, 1 set-up barrier passed, 2 results written (before the
// final barrier), 3 exit; 4 the SM; globaltimer nanoseconds, so CTAs on different SMs compare.
constexpr int kTraceCtas = 1024;
__device__ unsigned long long g_cta_trace[kTraceCtas][5];
#define RK_CTA_TRACE(event)                                                            \
    do {                                                                               \
        if (threadIdx.x == 0 && blockIdx.x < kTraceCtas) {                             \
            unsigned long long now;                                                    \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));                    \
            g_cta_trace[blockIdx.x][(event)] = now;                                    \
            if ((event) == 0) {                                                        \
                unsigned sm;                                                           \
                asm volatile("mov.u32 %0, %%smid;" : "=r"(sm));                        \
                g_cta_trace[blockIdx.x][4] = sm;                                       \
            }                                                                          \
        }                                                                              \
    } while (0)
#else
#define RK_CTA_TRACE(event) \
    do {                   \
    } while (0)
#define RK_WARP_TRACE(tile_index, event) \
    do {                                \
    } while (0)
#define RK_TRACE(tile_index, event) \
    do {                           \
    } while (0)
#endif

#ifdef RK_WAIT_TEST
// Wait-test build only: the key tile whose TMA loads CTA 0's producer never issues (-1: none), so
// that every wait on it runs out (set by rocmkernels_attention_test_withhold_tile).
__device__ int g_withheld_tile = -1;
#endif

constexpr int kQTile = 128;
constexpr int kKeyTile = 64;
constexpr float kPScale = 16384.f;  // P is split as P * 2^14
constexpr int kNoExponent = 1000;   // outside every clamped scale exponent
constexpr uint32_t kIdescS = f16_instr_desc(128, 64);  // S: 64 keys
constexpr uint64_t kDescStep = 2;                      // one K=16 step of FP16 = 32 bytes

// Configuration per storage mode and head width. Split FP32 (kHalf false): d = 32 has two Q tiles
// of 128 queries per CTA sharing each K/V tile (12 warps, 4 stages), or one Q tile (8 warps) when
// that grid fits in one wave of CTAs (launch below); d = 64 one Q tile per CTA (8 warps,
// 3 stages) with operands twice as wide. FP16 storage (kHalf true, d = 16, 32 or 64): one Q tile,
// 3 stages, one FP16 term per operand. The TMEM column layout of a Q tile is the same for one or
// two Q tiles.
// kPrepared (split FP32, d = 32): K and V arrive already split, as the stage images that
// prepare_kv_kernel wrote once per head (below); the CTA then has no split warps, and one MMA warp
// per Q tile instead of one for both.
// kRowThreads = 2 (prepared, one Q tile): two softmax threads per query row, each taking half of
// every key tile and half of the output columns (8 softmax warps per Q tile), and two CTAs per SM.
template <int D, bool kHalf, int kTiles = !kHalf && D == 32 ? 2 : 1, bool kPrepared = false, int kRowThreads = 1>
struct Forward {
    static_assert(kTiles == 1 || (kTiles == 2 && !kHalf && D == 32), "two Q tiles per CTA: split FP32, d = 32");
    static_assert(!kPrepared || (!kHalf && D == 32), "prepared operands: split FP32, d = 32");
    static_assert(kRowThreads == 1 || (kRowThreads == 2 && kPrepared && kTiles == 1), "two threads per row: prepared, one Q tile");
    static constexpr int kTerms = kHalf ? 1 : 2;  // FP16 terms per operand
    static constexpr int kQTiles = kTiles;
    static constexpr int kCtaQueries = kQTile * kQTiles;
    static constexpr int kStages = !kHalf && D == 32 ? 4 : 3;
    static constexpr int kSoftmaxWarps = 4 * kQTiles * kRowThreads;
    static constexpr int kMmaWarps = kPrepared ? kQTiles : 1, kSplitWarps = kPrepared ? 0 : 2;
    static constexpr int kProducerWarp = kSoftmaxWarps, kMmaWarp = kSoftmaxWarps + 1, kSplitWarp = kMmaWarp + kMmaWarps;
    static constexpr int kThreads = 32 * (kSoftmaxWarps + 1 + kMmaWarps + kSplitWarps);
    static constexpr int kSplitThreads = 64;
    // d = 64: the raw K/V stage is refilled as soon as the split warps have read it into registers
    // (their conversion then waits for the MMAs to release the converted stage). Measured on B200:
    // d = 64 171 -> 164 us (B8 H6 S1024); d = 32 slower (36.9 -> 39.9 us at B8 H3 S1024, 608 -> 674
    // at B4 H12 S4096: the two d = 32 split warps then run inside the softmax warps' busy phase on
    // the two sub-partitions they share), so d = 32 refills a stage after its MMAs finished.
    static constexpr bool kEarlyRawRefill = !kHalf && D == 64;
    static constexpr int kBoxes = kHalf ? 1 : D / 32;        // TMA boxes of 64 rows x 128 bytes per raw tile
    static constexpr int kRawFloats = kBoxes * kBoxFloats;  // raw tile of 64 keys in 32-bit words
    static constexpr int kKWords = kHalf ? 0 : 64 * D;       // row layout [k0 | k1] of 64 keys (FP16: the raw tile)
    static constexpr int kVRows = kHalf ? D : 2 * D + 16;    // B of P.V: v0^T, v1^T and 16 rows of ones (row sums);
                                                             // FP16: v^T only
    static constexpr int kVWords = kVRows * 32;              // kVRows x 128 bytes
    // TMEM per Q tile: q0 pairs | q1 pairs | S/P buffer 0 | S/P buffer 1 | Oa | Ob | row sums
    // (prepared operands: one output accumulator Ot, then the row sums)
    static constexpr uint32_t kColQ0 = 0, kColQ1 = D / 2, kColBuffer = kHalf ? 32 : D, kBufferColumns = 64,
                              kColO = kColBuffer + 128, kColSum = kColO + (kPrepared ? D : kTerms * D),
                              kColTile = kHalf || D == 32 ? 256 : 512;
    // One prepared Q tile uses 208 columns: 256, so that two such CTAs share an SM's TMEM.
    static constexpr uint32_t kTmemColumns = kHalf || (kPrepared && kQTiles == 1) ? 256 : 512;
    static constexpr uint64_t kDescStageK = (kHalf ? kRawFloats : kKWords) * 4 / 16, kDescStageV = kVWords * 4 / 16;
};

// Per key tile: which of its 64 keys are visible and the power-of-two scales of its split K and V
// (16 bytes, so that a bulk copy can land it beside a prepared stage image).
struct alignas(16) StageHeader {
    uint32_t mask[2];  // bit c of mask[c / 32]: key k0 + c visible
    int k_exponent;    // K tile scaled by 2^k_exponent
    int v_exponent;    // V tile scaled by 2^v_exponent
};

// A prepared stage image in global memory: the k16 tile (64 rows [k0 | k1], 8 KB) followed by the
// v1^T / v0^T rows of the vt16 tile (64 rows of 128 bytes), byte for byte as the shared-memory
// stage holds them.
constexpr int kImageKBytes = 64 * 2 * 32 * 2, kImageBytes = kImageKBytes + 64 * 128;

// Operand tiles are rows of 128 bytes in 1024-byte aligned 8-row atoms (the 128B swizzle).
template <int D, bool kHalf, int kTiles = Forward<D, kHalf>::kQTiles, bool kPrepared = false, int kRowThreads = 1>
struct alignas(1024) SharedStorage {
    using F = Forward<D, kHalf, kTiles, kPrepared, kRowThreads>;
    // Raw tiles as TMA lands them (FP32: swizzled boxes of 64 x 32; FP16: 64 x 64); prepared
    // operands have none (a 1 KB placeholder keeps the layout below aligned).
    static constexpr int kRawStages = kPrepared ? 1 : F::kStages, kRawWords = kPrepared ? 256 : F::kRawFloats;
    float k_raw[kRawStages][kRawWords];        // K tile
    float v_raw[kRawStages][kRawWords];        // V tile
    uint32_t k16[F::kStages][F::kKWords > 0 ? F::kKWords : 1];  // 64 key rows as [k0 | k1] FP16 (row layout),
                                                                // K-major 128B swizzle (unused for FP16 storage)
    alignas(1024) uint32_t vt16[F::kStages][F::kVWords];  // rows 0..D-1 v0^T, D..2D-1 v1^T (64 keys each, 128B
                                                          // swizzle), 2D..2D+15 FP16 ones (written once); FP16: v^T
    StageHeader header[F::kStages];            // the stage's key mask and exponents
    float split_max[2][2];                     // per split warp: max |K|, max |V| of its rows
    int split_ok[2];                           // per split warp: its kv_full wait succeeded
    uint64_t kv_full[F::kStages];              // TMA bytes landed
    uint64_t raw_free[F::kStages];             // kEarlyRawRefill: the raw tiles read by the split warps (64 arrivals)
    uint64_t kv_ready[F::kStages];             // conversion done (64 arrivals)
    uint64_t kv_empty[F::kStages];             // MMAs reading the stage finished (a commit per MMA warp)
    uint64_t s_full[F::kQTiles][2];            // S of a buffer is in TMEM (commit)
    uint64_t p_full[F::kQTiles];               // P of the current tile is in TMEM (128 arrivals)
    uint64_t pv_done[F::kQTiles];              // Ot of the current tile is in TMEM (commit)
    uint64_t q_ready;                          // q0/q1 of every Q tile in TMEM (128 arrivals per tile and row thread)
    // kRowThreads = 2: each thread's partial row max of a tile, [tile parity][half][row], and per
    // lane quarter the barrier the quarter's two warps meet at once both halves are written.
    float row_exchange[kRowThreads == 2 ? 2 : 1][kRowThreads][kRowThreads == 2 ? kQTile : 1];
    uint64_t pair_bar[kRowThreads == 2 ? 4 : 1];
    uint64_t range_ready;                      // tile_count written (1 arrival)
    int tile_count;                            // key tiles up to the last visible key of the window
    uint64_t mma_done;                         // every MMA of the CTA finished (a commit per MMA warp)
    uint32_t tmem_base;
};

// The rotary prologue's extra operands: per stage, the cos and sin rows of the tile's 64 keys as
// TMA lands them (64 rows x 32 FP32, 128B swizzle, the layout of one K box).
template <int D, int kTiles>
struct alignas(1024) RotaryStorage : SharedStorage<D, false, kTiles> {
    alignas(1024) float cos_raw[Forward<D, false>::kStages][kBoxFloats];
    alignas(1024) float sin_raw[Forward<D, false>::kStages][kBoxFloats];
};

struct FlashArgs {
    AttentionParams p;
    int cta_per_head;  // ceil(queries / queries per CTA)
    int vec_out;       // output rows 16-byte addressable
    int rot_batch;     // rotary tables: 1 = one table per sequence (batch coordinate b), 0 = one shared table
    // Prepared operands: the stage images and headers of key tile t of head (b, h) at index
    // (b * heads + h) * tiles_per_head + t.
    const uint8_t *images;
    const StageHeader *headers;
    int tiles_per_head;
};

__device__ __forceinline__ uint32_t tmem_lane_address(uint32_t base, int warp) {
    return base + (static_cast<uint32_t>((warp & 3) * 32) << 16);
}

// S(buffer) = q0.k1 + q1.k0 + q0.k0 over the D features (D/16 K=16 steps each), then a commit to
// `bar`; k_desc addresses the stage's k16 tile. FP16 storage: S = q.k, k_desc addressing the raw
// K tile. Warp-collective.
template <int D, bool kHalf>
__device__ __forceinline__ void issue_scores(uint32_t tmem, uint64_t k_desc, int tile, int buffer, uint64_t *bar) {
    using F = Forward<D, kHalf>;
    const uint32_t t = tmem + tile * F::kColTile;
    const uint32_t d = t + F::kColBuffer + buffer * F::kBufferColumns;
    const uint32_t a0 = t + F::kColQ0, a1 = t + F::kColQ1;
    if constexpr (kHalf) {
        if constexpr (D == 16) {
            mma1_f16_ts_commit_warp(d, a0, k_desc, kIdescS, 1, bar);
        } else if constexpr (D == 32) {
            mma2_f16_ts_first_commit_warp(d, a0, a0 + 8, k_desc, k_desc + kDescStep, kIdescS, 1, bar);
        } else {
            const uint32_t a[4] = {a0, a0 + 8, a0 + 16, a0 + 24};
            const uint64_t bk[4] = {k_desc, k_desc + kDescStep, k_desc + 2 * kDescStep, k_desc + 3 * kDescStep};
            mma4_f16_ts_commit_warp(d, a, bk, kIdescS, 1, bar);
        }
        return;
    }
    constexpr uint64_t x1 = row_x1_offset<D>();
    if constexpr (D == 32) {
        const uint32_t a[4] = {a0, a0 + 8, a1, a1 + 8};
        const uint64_t bk[4] = {k_desc + x1, k_desc + x1 + kDescStep, k_desc, k_desc + kDescStep};
        mma4_f16_ts_warp(d, a, bk, kIdescS, 1);
        mma2_f16_ts_commit_warp(d, a0, a0 + 8, k_desc, k_desc + kDescStep, kIdescS, bar);
    } else {
        const uint32_t g1a[4] = {a0, a0 + 8, a0 + 16, a0 + 24};  // q0 . k1
        const uint64_t g1b[4] = {k_desc + x1, k_desc + x1 + kDescStep, k_desc + x1 + 2 * kDescStep, k_desc + x1 + 3 * kDescStep};
        mma4_f16_ts_warp(d, g1a, g1b, kIdescS, 1);
        const uint32_t g2a[4] = {a1, a1 + 8, a1 + 16, a1 + 24};  // q1 . k0
        const uint64_t g2b[4] = {k_desc, k_desc + kDescStep, k_desc + 2 * kDescStep, k_desc + 3 * kDescStep};
        mma4_f16_ts_warp(d, g2a, g2b, kIdescS, 0);
        mma4_f16_ts_commit_warp(d, g1a, g2b, kIdescS, 0, bar);  // q0 . k0
    }
}

// [Oa | Ob | sums] = p1.[v0 ; v1 ; 1] + p0.[v0 ; v1 ; 1] over the 64 keys (four K=16 steps
// each), then a commit to `bar`; v_desc addresses the stage's vt16 tile. FP16 storage:
// [O | sums] = p.[v ; 1]. Warp-collective.
template <int D, bool kHalf>
__device__ __forceinline__ void issue_values(uint32_t tmem, uint64_t v_desc, int tile, int buffer, uint64_t *bar) {
    using F = Forward<D, kHalf>;
    const uint32_t t = tmem + tile * F::kColTile;
    const uint32_t pbuf = t + F::kColBuffer + buffer * F::kBufferColumns;
    constexpr uint32_t kIdescPV = f16_instr_desc(128, F::kVRows);
    const uint64_t bv[4] = {v_desc, v_desc + kDescStep, v_desc + 2 * kDescStep, v_desc + 3 * kDescStep};
    const uint32_t a0[4] = {pbuf, pbuf + 8, pbuf + 16, pbuf + 24};
    if constexpr (!kHalf) {
        const uint32_t a1[4] = {pbuf + 32, pbuf + 40, pbuf + 48, pbuf + 56};
        mma4_f16_ts_warp(t + F::kColO, a1, bv, kIdescPV, 1);
    }
    mma4_f16_ts_commit_warp(t + F::kColO, a0, bv, kIdescPV, kHalf ? 1 : 0, bar);
}

// Prepared operands, d = 32: Ot = p1.v0 + p0.v1 + p0.v0 in one accumulator, and the row sums
// p1.1 + p0.1 beside it, over the 64 keys (four K=16 steps per product), then a commit to `bar`.
// The stage's V tile holds rows [v1^T ; v0^T ; ones]: B1 = v1^T (N = 32), B0 = [v0^T ; ones]
// (N = 48, 32 rows = 4 KB further). The two small products go in first, so the accumulator is
// small while they are added; the p1.v1 term (~2^-22 of the output) is left out.
template <int kTiles>
__device__ __forceinline__ void issue_values_prepared(uint32_t tmem, uint64_t v_desc, int tile, int buffer, uint64_t *bar) {
    using F = Forward<32, false, kTiles, true>;
    const uint32_t t = tmem + tile * F::kColTile;
    const uint32_t pbuf = t + F::kColBuffer + buffer * F::kBufferColumns;
    constexpr uint32_t kIdescOutSums = f16_instr_desc(128, 48), kIdescOut = f16_instr_desc(128, 32);
    constexpr uint64_t kRowsV0 = 32 * 128 / 16;  // descriptor offset of the v0^T rows
    const uint64_t b1[4] = {v_desc, v_desc + kDescStep, v_desc + 2 * kDescStep, v_desc + 3 * kDescStep};
    const uint64_t b0[4] = {v_desc + kRowsV0, v_desc + kRowsV0 + kDescStep, v_desc + kRowsV0 + 2 * kDescStep,
                            v_desc + kRowsV0 + 3 * kDescStep};
    const uint32_t a0[4] = {pbuf, pbuf + 8, pbuf + 16, pbuf + 24};       // p0 pairs
    const uint32_t a1[4] = {pbuf + 32, pbuf + 40, pbuf + 48, pbuf + 56};  // p1 pairs
    mma4_f16_ts_warp(t + F::kColO, a1, b0, kIdescOutSums, 1);
    mma4_f16_ts_warp(t + F::kColO, a0, b1, kIdescOut, 0);
    mma4_f16_ts_commit_warp(t + F::kColO, a0, b0, kIdescOutSums, 0, bar);
}

// Prepared operands, d = 32: folds a finished key tile's Ot (32 columns, V scaled by 2^c) and row
// sum into the running output and sum, with the same exponent rule as fold_output.
template <int N>
__device__ __forceinline__ void fold_prepared(float (&o)[N], float &row_sum, int &o_exp, const float (&ot)[N], float sum,
                                              float weight, int c) {
    if (o_exp == kNoExponent) o_exp = c;
    float out_weight = weight, tile_scale = 1.f;
    if (c > o_exp) {
        tile_scale = exp2_int(o_exp - c);
    } else if (c < o_exp) {
        out_weight = weight * exp2_int(c - o_exp);
        o_exp = c;
    }
    row_sum = fmaf(row_sum, weight, sum);
    const float2 weight2 = make_float2(out_weight, out_weight);
    if (__all_sync(0xffffffffu, tile_scale == 1.f)) {  // uniform anyway
#pragma unroll
        for (int i = 0; i < N; i += 2) {
            const float2 r = fma_f32x2(make_float2(o[i], o[i + 1]), weight2, make_float2(ot[i], ot[i + 1]));
            o[i] = r.x;
            o[i + 1] = r.y;
        }
    } else {
        const float2 scale2 = make_float2(tile_scale, tile_scale);
#pragma unroll
        for (int i = 0; i < N; i += 2) {
            const float2 u = mul_f32x2(make_float2(ot[i], ot[i + 1]), scale2);
            const float2 r = fma_f32x2(make_float2(o[i], o[i + 1]), weight2, u);
            o[i] = r.x;
            o[i + 1] = r.y;
        }
    }
}

// Folds the last finished key tile into the running output and row sum. In TMEM, Oa + Ob is the
// tile's P.V with V scaled by 2^c (c = the tile's V exponent) and the sum column its row sum of P.
// The running output is held as O * 2^o_exp, o_exp being the smallest V exponent folded so far:
// a tile with that exponent (the usual case, warp-uniform) costs one add and one FMA per column;
// a tile with another exponent moves whichever side has the larger one down, so no value is
// ever scaled up.
// FP16 storage has no exponents (c = o_exp = 0) and keeps its row sum itself: O = O * weight + Ot
// over the D columns.
template <int D, bool kHalf>
__device__ __forceinline__ void fold_output(float (&o)[D], float &row_sum, int &o_exp, uint32_t lane_base, float weight,
                                            int c) {
    using F = Forward<D, kHalf>;
    if constexpr (kHalf) {
        o_exp = 0;
        float ta[16], tb[16];
        if constexpr (D == 16)
            tmem_load16(lane_base + F::kColO, ta);
        else
            tmem_load16x2(lane_base + F::kColO, ta, lane_base + F::kColO + 16, tb);
#pragma unroll
        for (int i = 0; i < 16; ++i) o[i] = fmaf(o[i], weight, ta[i]);
        if constexpr (D >= 32) {
#pragma unroll
            for (int i = 0; i < 16; ++i) o[16 + i] = fmaf(o[16 + i], weight, tb[i]);
        }
        if constexpr (D == 64) {
            tmem_load16x2(lane_base + F::kColO + 32, ta, lane_base + F::kColO + 48, tb);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                o[32 + i] = fmaf(o[32 + i], weight, ta[i]);
                o[48 + i] = fmaf(o[48 + i], weight, tb[i]);
            }
        }
        return;
    }
    if (o_exp == kNoExponent) o_exp = c;
    float out_weight = weight, tile_scale = 1.f;
    if (c > o_exp) {
        tile_scale = exp2_int(o_exp - c);
    } else if (c < o_exp) {
        out_weight = weight * exp2_int(c - o_exp);
        o_exp = c;
    }
    float oa[16], ob[16], sum;
    tmem_load16x2_1(lane_base + F::kColO, oa, lane_base + F::kColO + D, ob, lane_base + F::kColSum, sum);
    row_sum = fmaf(row_sum, weight, sum);
    const bool unscaled = __all_sync(0xffffffffu, tile_scale == 1.f);  // uniform anyway
#pragma unroll
    for (int part = 0; part < D / 16; ++part) {
        if (part > 0) tmem_load16x2(lane_base + F::kColO + 16 * part, oa, lane_base + F::kColO + D + 16 * part, ob);
        const float2 weight2 = make_float2(out_weight, out_weight);
        if (unscaled) {
#pragma unroll
            for (int i = 0; i < 16; i += 2) {
                const float2 t = add_f32x2(make_float2(oa[i], oa[i + 1]), make_float2(ob[i], ob[i + 1]));
                const float2 r = fma_f32x2(make_float2(o[16 * part + i], o[16 * part + i + 1]), weight2, t);
                o[16 * part + i] = r.x;
                o[16 * part + i + 1] = r.y;
            }
        } else {
            const float2 scale2 = make_float2(tile_scale, tile_scale);
#pragma unroll
            for (int i = 0; i < 16; i += 2) {
                const float2 t = add_f32x2(make_float2(oa[i], oa[i + 1]), make_float2(ob[i], ob[i + 1]));
                const float2 u = mul_f32x2(t, scale2);
                const float2 r = fma_f32x2(make_float2(o[16 * part + i], o[16 * part + i + 1]), weight2, u);
                o[16 * part + i] = r.x;
                o[16 * part + i + 1] = r.y;
            }
        }
    }
}

// P' = 2^14 exp(S - max) = exp2(S * slope + offset) of 64 scores, split into FP16 pairs: p0 =
// P' truncated to 11 significant bits (exact in FP16), p1 = FP16(P' - p0), stored to the P
// buffer (p0 pairs in columns 0-31, p1 pairs in 32-63) in chunks of 16 keys without waiting, so
// few values are live at a time. kPlain: every score is finite or -inf and the offset is finite,
// so exp2(-inf) = 0 covers the masked keys; otherwise -inf scores are zeroed explicitly (a row
// without any visible key yet has an infinite offset). kHalf: P' rounded to FP16 once, pairs in
// columns 0-31, and the FP32 sum of the unrounded P' returned (0 otherwise).
// kPacked: the exponent arguments and residuals as packed FP32 pairs (fma/sub .f32x2: one issue
// for two values). Used where registers allow: the split d = 32 kernel with two Q tiles (168
// registers a thread) spills with it and is faster without (36.9 against 36.2 us at B8 H3 S1024);
// d = 64 gains 8 %, the one-Q-tile d = 32 kernel 6-7 %.
// kValues = 32 (two threads per row): the 32 scores of this thread's half of the tile; pbuf then
// addresses its 16 p0 columns (its p1 columns follow 32 columns further, as for a whole row).
template <bool kPlain, bool kHalf, bool kPacked, int kValues = 64>
__device__ __forceinline__ float exp_split_store(const float (&sc)[kValues], float slope, float offset, uint32_t pbuf) {
    float sum[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int chunk = 0; chunk < kValues / 16; ++chunk) {
        float p0[8], p1[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int c = 8 * chunk + i;
            float a, b;
            if constexpr (kPacked) {
                const float2 arg = fma_f32x2(make_float2(sc[2 * c], sc[2 * c + 1]), make_float2(slope, slope), make_float2(offset, offset));
                a = fast_exp2(arg.x);
                b = fast_exp2(arg.y);
            } else {
                a = fast_exp2(fmaf(sc[2 * c], slope, offset));
                b = fast_exp2(fmaf(sc[2 * c + 1], slope, offset));
            }
            if (!kPlain) {
                a = sc[2 * c] == -INFINITY ? 0.f : a;
                b = sc[2 * c + 1] == -INFINITY ? 0.f : b;
            }
            if constexpr (kHalf) {
                p0[i] = __uint_as_float(pack_half2(a, b));
                sum[i & 3] += a + b;
            } else {
                const float a0 = __uint_as_float(__float_as_uint(a) & 0xFFFFE000u);
                const float b0 = __uint_as_float(__float_as_uint(b) & 0xFFFFE000u);
                p0[i] = __uint_as_float(pack_half2(a0, b0));
                if constexpr (kPacked) {
                    const float2 residual = sub_f32x2(make_float2(a, b), make_float2(a0, b0));
                    p1[i] = __uint_as_float(pack_half2(residual.x, residual.y));
                } else {
                    p1[i] = __uint_as_float(pack_half2(a - a0, b - b0));
                }
            }
        }
        if constexpr (kHalf)
            tmem_store8_async(pbuf + 8 * chunk, p0);
        else
            tmem_store8x2_async(pbuf + 8 * chunk, p0, pbuf + 32 + 8 * chunk, p1);
    }
    return (sum[0] + sum[1]) + (sum[2] + sum[3]);
}

// V tile -> V^T operand rows for FP16 storage. Split warp w transposes the key groups 4w..4w+3
// (its own 32 rows, whose mask bits are `bits`); lane -> (group g = 4w + lane % 4, feature chunk
// fc = lane / 4 < D / 8): the 8 x 8 FP16 block of rows 8g..8g+7 and features 8fc..8fc+7, masked
// rows zeroed, becomes chunk g of the V^T rows 8fc..8fc+7 (pairs regrouped with byte permutes).
template <int D>
__device__ __forceinline__ void transpose_values(const float *v_raw, uint32_t *vt16, int w, int lane, uint32_t bits) {
    const int fc = lane >> 2;
    if (fc >= D / 8) return;
    const int g = 4 * w + (lane & 3);
    const uint4 *raw = reinterpret_cast<const uint4 *>(v_raw);
    uint32_t x[8][4];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
        const int vrow = 8 * g + r;
        uint4 chunk = raw[vrow * 8 + (fc ^ (vrow & 7))];
        if (!((bits >> (vrow & 31)) & 1)) chunk = make_uint4(0u, 0u, 0u, 0u);
        x[r][0] = chunk.x;
        x[r][1] = chunk.y;
        x[r][2] = chunk.z;
        x[r][3] = chunk.w;
    }
    uint4 *vt = reinterpret_cast<uint4 *>(vt16);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        const uint32_t select = (e & 1) ? 0x7632u : 0x5410u;  // high or low halves of two words
        const int f = 8 * fc + e;
        vt[f * 8 + (g ^ (f & 7))] = make_uint4(__byte_perm(x[0][e >> 1], x[1][e >> 1], select),
                                               __byte_perm(x[2][e >> 1], x[3][e >> 1], select),
                                               __byte_perm(x[4][e >> 1], x[5][e >> 1], select),
                                               __byte_perm(x[6][e >> 1], x[7][e >> 1], select));
    }
}

// Rotary prologue of a 32-wide FP32 row held as 8 float4 (features 4c..4c+3 in x[c]): features f
// and f + 16 rotate by the row's tables cs, sn (same layout; rotate_pair, the rotary_fp32 forward).
__device__ __forceinline__ void rotate_row32(float4 (&x)[8], const float4 (&cs)[8], const float4 (&sn)[8]) {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const float4 cl = cs[c], ch = cs[c + 4], sl = sn[c], sh = sn[c + 4];
        float4 &lo = x[c], &hi = x[c + 4];
        rotate_pair<false>(lo.x, hi.x, cl.x, ch.x, sl.x, sh.x, lo.x, hi.x);
        rotate_pair<false>(lo.y, hi.y, cl.y, ch.y, sl.y, sh.y, lo.y, hi.y);
        rotate_pair<false>(lo.z, hi.z, cl.z, ch.z, sl.z, sh.z, lo.z, hi.z);
        rotate_pair<false>(lo.w, hi.w, cl.w, ch.w, sl.w, sh.w, lo.w, hi.w);
    }
}

// kWidth: the tensors' head width when it is below the kernel's D (FP32 storage with 16 features
// on the D = 32 kernel): the tensor maps are kWidth wide, so the TMA fills features kWidth..D-1
// of K and V with zeros, Q rows are read and O rows written kWidth wide.
// kRotary (D = 32, FP32): the rotary prologue — each Q row (softmax threads) and each K row (split
// warps) is rotated by its token's tables before it is scaled and split, so the rotated tensors
// never go through HBM; the result equals rotary_fp32 followed by this kernel bit for bit.
// With kRotary the producer also lands the tile's cos and sin rows (tmap_cos, tmap_sin) in the
// stage; the other instantiations ignore those two maps.
// kPrepared (D = 32, split FP32, no statistics): the key tiles come from the stage images of
// prepare_kv_kernel (args.images / args.headers; with kRotary its K rows are already rotated and
// the kernel rotates only the Q rows) by bulk copies, and the kernel is launched as a programmatic
// dependent of that pre-pass: the producer thread passes griddepcontrol.wait before its first copy,
// while the other threads allocate TMEM, set up the barriers and split their Q rows.
// kChained: launched as a programmatic dependent of the grid before it in the stream (one-wave
// one-tile grids only, below): the next grid may be scheduled at once, TMEM is allocated while
// the grid ahead still runs, and nothing in global memory is touched before that grid completed.
template <int D, bool kHalf, int kWidth = D, bool kRotary = false, int kTiles = Forward<D, kHalf>::kQTiles,
          bool kStats = false, bool kPrepared = false, int kRowThreads = 1, bool kChained = false>
__global__ void __launch_bounds__(Forward<D, kHalf, kTiles, kPrepared, kRowThreads>::kThreads, kRowThreads == 2 ? 2 : 1)
        flash_forward_kernel(const FlashArgs args, const __grid_constant__ CUtensorMap tmap_k,
                             const __grid_constant__ CUtensorMap tmap_v, const __grid_constant__ CUtensorMap tmap_cos,
                             const __grid_constant__ CUtensorMap tmap_sin) {
    static_assert(kWidth == D || (!kHalf && kWidth % 4 == 0 && kWidth < D), "narrow rows: FP32 storage only");
    static_assert(!kRotary || (D == 32 && kWidth == 32 && !kHalf), "the rotary prologue is defined for 32-wide FP32 heads");
    static_assert(!kStats || (D == 32 && kWidth == 32 && !kHalf && !kRotary), "statistics: 32-wide FP32 heads");
    static_assert(!kPrepared || (D == 32 && kWidth == 32 && !kHalf && !kStats), "prepared operands: the d = 32 split-FP32 forward");
    static_assert(!kChained || !kPrepared, "the prepared forward is already its pre-pass's dependent");
    using F = Forward<D, kHalf, kTiles, kPrepared, kRowThreads>;
    // Prepared operands with the rotary prologue: K arrives rotated, so no table tiles are staged.
    using Storage = std::conditional_t<kRotary && !kPrepared, RotaryStorage<D, kTiles>,
                                       SharedStorage<D, kHalf, kTiles, kPrepared, kRowThreads>>;
    constexpr int kStages = F::kStages;
    extern __shared__ uint8_t shared_raw[];
    Storage &s = *reinterpret_cast<Storage *>((reinterpret_cast<uintptr_t>(shared_raw) + 1023) & ~uintptr_t(1023));
    const AttentionParams &p = args.p;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    RK_CTA_TRACE(0);

    int block = blockIdx.x;
    const int cta_tile = block % args.cta_per_head;
    block /= args.cta_per_head;
    const int h = block % p.heads;
    const int b = block / p.heads;
    const int q0 = cta_tile * F::kCtaQueries;
    int first, last;
    key_window(q0, min(q0 + F::kCtaQueries, p.queries), p.keys, p.radius, first, last);
    // Prepared images cover the fixed 64-key tiles of the sequence: the window starts on one (the
    // keys before the true start are outside every row's radius and drop out with the window mask).
    if constexpr (kPrepared) first &= ~(kKeyTile - 1);
    // Key tiles of the window; trailing tiles whose keys are all masked are dropped after the
    // set-up barrier (visible_tiles below), so that key-padded sequences skip their padding.
    const int window_tiles = last > first ? (last - first + kKeyTile - 1) / kKeyTile : 0;

    if constexpr (kPrepared || kChained) {
        if constexpr (kChained) grid_launch_dependents();
        if (warp == 0) {
            tmem_alloc(&s.tmem_base, F::kTmemColumns);
            tmem_relinquish();
        }
        if constexpr (kChained) grid_dependency_wait();
    }
    // The softmax threads issue the loads of their Q row (and, with the rotary prologue, of its
    // table rows) before the set-up barrier, so their latency overlaps the TMEM allocation and
    // the barrier initialisation.
    constexpr int kQChunks = kHalf ? D / 8 : D / 4;  // 16-byte chunks of a Q row
    uint4 q_chunks[kQChunks];
    float4 q_cos[kRotary ? 8 : 1], q_sin[kRotary ? 8 : 1];
    const int query = q0 + (kRowThreads == 2 ? 0 : warp >> 2) * kQTile + (threadIdx.x & (kQTile - 1));  // softmax threads' row
    const bool row_valid = warp < F::kSoftmaxWarps && query < p.queries;
    {
        const uint4 *src = kHalf ? reinterpret_cast<const uint4 *>(p.q.row_as<__half>(b, h, row_valid ? query : 0))
                                 : reinterpret_cast<const uint4 *>(p.q.row(b, h, row_valid ? query : 0));
#pragma unroll
        for (int c = 0; c < kQChunks; ++c)
            q_chunks[c] = row_valid && (kHalf || c < kWidth / 4) ? __ldg(src + c) : make_uint4(0u, 0u, 0u, 0u);
        if constexpr (kRotary) {
            const float4 *c4 = reinterpret_cast<const float4 *>(p.cos_row(b, row_valid ? query : 0));
            const float4 *s4 = reinterpret_cast<const float4 *>(p.sin_row(b, row_valid ? query : 0));
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                q_cos[c] = row_valid ? __ldg(c4 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
                q_sin[c] = row_valid ? __ldg(s4 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
    }

    if (!kPrepared && !kChained && warp == 0) {
        tmem_alloc(&s.tmem_base, F::kTmemColumns);
        tmem_relinquish();
    }
    // TMA loads of key tile j into its stage, completing on kv_full (producer thread only).
    // Prepared operands: bulk copies of the tile's stage image and header.
    const auto issue_tile = [&](int j) {
        const int stage = j % kStages;
#ifdef RK_WAIT_TEST
        if (blockIdx.x == 0 && j == g_withheld_tile) return;  // its kv_full phase never completes
#endif
        RK_TRACE(j, 12);
        if constexpr (kPrepared) {
            const long long tile = (static_cast<long long>(b) * p.heads + h) * args.tiles_per_head + first / kKeyTile + j;
            const uint8_t *image = args.images + tile * kImageBytes;
            mbar_arrive_expect_tx(&s.kv_full[stage], kImageBytes + sizeof(StageHeader));
            bulk_load(s.k16[stage], image, kImageKBytes, &s.kv_full[stage]);
            bulk_load(s.vt16[stage], image + kImageKBytes, kImageBytes - kImageKBytes, &s.kv_full[stage]);
            bulk_load(&s.header[stage], args.headers + tile, sizeof(StageHeader), &s.kv_full[stage]);
            return;
        }
        mbar_arrive_expect_tx(&s.kv_full[stage], ((kStats ? 1 : 2) * F::kBoxes + (kRotary ? 2 : 0)) * kBoxBytes);
        if constexpr (kRotary && !kPrepared) {
            const int table = b * args.rot_batch;
            tma_load_4d(s.cos_raw[stage], &tmap_cos, &s.kv_full[stage], 0, first + j * kKeyTile, 0, table);
            tma_load_4d(s.sin_raw[stage], &tmap_sin, &s.kv_full[stage], 0, first + j * kKeyTile, 0, table);
        }
#pragma unroll
        for (int box = 0; box < F::kBoxes; ++box) {
            tma_load_4d(s.k_raw[stage] + box * kBoxFloats, &tmap_k, &s.kv_full[stage], 32 * box, first + j * kKeyTile, h, b);
            if constexpr (!kStats)
                tma_load_4d(s.v_raw[stage] + box * kBoxFloats, &tmap_v, &s.kv_full[stage], 32 * box, first + j * kKeyTile, h, b);
        }
    };
    const int prefetched = min(window_tiles, kStages);  // issued before the set-up barrier
    if (threadIdx.x == F::kProducerWarp * 32) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&s.kv_full[i], 1);
            mbar_init(&s.raw_free[i], F::kSplitThreads);
            mbar_init(&s.kv_ready[i], F::kSplitThreads);
            mbar_init(&s.kv_empty[i], F::kMmaWarps);
        }
        for (int t = 0; t < F::kQTiles; ++t) {
            mbar_init(&s.s_full[t][0], 1);
            mbar_init(&s.s_full[t][1], 1);
            mbar_init(&s.p_full[t], kQTile * kRowThreads);
            mbar_init(&s.pv_done[t], 1);
        }
        mbar_init(&s.q_ready, kQTile * F::kQTiles * kRowThreads);
        if constexpr (kRowThreads == 2) {
            for (int quarter = 0; quarter < 4; ++quarter) mbar_init(&s.pair_bar[quarter], 64);
        }
        mbar_init(&s.range_ready, 1);
        mbar_init(&s.mma_done, F::kMmaWarps);
        mbar_fence_init();
        // Prepared operands: the stage images are the pre-pass's output, the one thing this grid
        // reads that the grid before it writes (its other inputs were written before the pre-pass
        // started), so only this thread waits for the pre-pass, right before its first copy.
        if constexpr (kPrepared) grid_dependency_wait();
        // The first stages are free: their loads overlap the TMEM allocation and the set-up
        // barrier. Nothing else touches the raw K/V tiles or kv_full before that barrier.
        for (int j = 0; j < prefetched; ++j) issue_tile(j);
    }
    // Rows 2D..2D+15 of every V operand tile are FP16 ones, so P.V also yields the row sums of P.
    if constexpr (!kHalf) {
        for (int i = threadIdx.x; i < kStages * 16 * 32; i += F::kThreads)
            s.vt16[i / (16 * 32)][2 * D * 32 + i % (16 * 32)] = 0x3C003C00u;
    }
    fence_proxy_async_shared();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    RK_CTA_TRACE(1);
    const uint32_t tmem = s.tmem_base;
    // The window's tiles up to its last visible key (published by the producer warp).
    const auto visible_tiles = [&]() { return mbar_wait(&s.range_ready, 0) ? s.tile_count : 0; };

    if (warp == F::kProducerWarp) {
        // ---------------------------------------------------------------- TMA producer
        // The last visible key of the window: the mask read backwards 128 keys at a time (one
        // step when the window's last keys are visible), while the first tiles' loads are in
        // flight.
        const int tiles = visible_tiles_of(p.mask + static_cast<long long>(b) * p.keys, first, last, lane);
        if (lane == 0) {
            s.tile_count = tiles;
            mbar_arrive(&s.range_ready);
            int issued = prefetched;
            bool ok = true;
            for (int j = prefetched; j < tiles && ok; ++j) {
                const int stage = j % kStages, use = j / kStages;
                // j >= kStages here. kEarlyRawRefill: the raw stage is free once the split warps
                // have read tile j - kStages into registers (the MMAs read only the converted
                // tiles); otherwise once the MMAs reading the stage finished.
                ok = mbar_wait(F::kEarlyRawRefill ? &s.raw_free[stage] : &s.kv_empty[stage], (use - 1) & 1);
                if (!ok) break;
                issue_tile(j);
                ++issued;
            }
            // No copy may still be in flight into the shared memory of a finishing CTA. The last
            // use of each stage is waited for even when every wait above succeeded: if the split
            // warps gave up, the MMA warp still releases the stages it had, and the tiles issued
            // into them are consumed by nobody. On the normal path these phases completed long
            // ago (the split warps waited for them), so each wait is one test.
            for (int j = max(0, issued - kStages); j < issued; ++j) mbar_wait(&s.kv_full[j % kStages], (j / kStages) & 1);
            // Prefetched tiles past the last visible key are never converted: wait for them.
            for (int j = tiles; j < prefetched; ++j) mbar_wait(&s.kv_full[j], 0);
        }
    } else if (kPrepared && warp >= F::kMmaWarp && warp < F::kMmaWarp + F::kMmaWarps) {
        // ---------------------------------------------------------------- MMA issuers (prepared operands)
        // Warp kMmaWarp + t issues Q tile t's products: S(t, 0) and S(t, 1) first; then for every
        // key tile j, once P(t, j) is in TMEM, P(t, j).V (the stage's release follows it) and
        // S(t, j + 2) into the buffer P(t, j) occupies (the tensor core runs one thread's MMAs in
        // order, so S(t, j + 2) overwrites P(t, j) only after P(t, j).V has read it). Every wait
        // suspends the warp, so it takes no issue slots from the softmax warps of its sub-partition.
        const int t = warp - F::kMmaWarp;
        const int tiles = __shfl_sync(0xffffffffu, visible_tiles(), 0);
        if (tiles > 0) {
            const uint64_t k_desc0 = sw128_descriptor(smem_u32(s.k16[0]));
            const uint64_t v_desc0 = sw128_descriptor(smem_u32(s.vt16[0]));
            bool ok = mbar_wait_sleep_warp(&s.q_ready, 0);
            tc_fence_after();
            for (int j = 0; j < min(2, tiles) && ok; ++j) {
                ok = mbar_wait_sleep_warp(&s.kv_full[j], 0);
                if (!ok) break;
                tc_fence_after();
                issue_scores<D, kHalf>(tmem, k_desc0 + F::kDescStageK * j, t, j, &s.s_full[t][j]);
            }
            for (int j = 0; j < tiles && ok; ++j) {
                const int stage = j % kStages, buffer = j & 1;
                if (lane == 0) RK_TRACE(j, 2 + t);
                ok = mbar_wait_sleep_warp(&s.p_full[t], j & 1);
                if (!ok) break;
                if (lane == 0) RK_TRACE(j, t);
                tc_fence_after();
                issue_values_prepared<kTiles>(tmem, v_desc0 + F::kDescStageV * stage, t, buffer, &s.pv_done[t]);
                mma_commit_warp(&s.kv_empty[stage]);
                if (lane == 0) RK_TRACE(j, 13 + t);
                if (j + 2 < tiles) {
                    const int next = (j + 2) % kStages;
                    ok = mbar_wait_sleep_warp(&s.kv_full[next], ((j + 2) / kStages) & 1);
                    if (!ok) break;
                    tc_fence_after();
                    issue_scores<D, kHalf>(tmem, k_desc0 + F::kDescStageK * next, t, buffer, &s.s_full[t][buffer]);
                    if (lane == 0) RK_TRACE(j, 7 + 4 * t);
                }
            }
            // TMEM is released only after every issued MMA of both warps has completed.
            mma_commit_warp(&s.mma_done);
            mbar_wait_warp(&s.mma_done, 0);
        }
    } else if (!kPrepared && warp == F::kMmaWarp) {
        // ---------------------------------------------------------------- MMA issuer
        // S(t, 0) and S(t, 1) first; then for every key tile j, whichever Q tile's P is ready
        // first gets P(j).V and S(j + 2) (into the buffer P(j) occupied) issued first; the K/V
        // stage of tile j is released once every P.V product is issued. The whole warp runs
        // the loop (uniform control flow and descriptors); elected lanes issue the tcgen05 ops.
        const int tiles = __shfl_sync(0xffffffffu, visible_tiles(), 0);
        if (tiles > 0) {
            const uint64_t k_desc0 = sw128_descriptor(smem_u32(kHalf ? static_cast<const void *>(s.k_raw[0]) : s.k16[0]));
            const uint64_t v_desc0 = sw128_descriptor(smem_u32(s.vt16[0]));
            bool ok = mbar_wait_warp(&s.q_ready, 0);
            tc_fence_after();
            for (int j = 0; j < min(2, tiles) && ok; ++j) {
                ok = mbar_wait_warp(&s.kv_ready[j], 0);
                tc_fence_after();
                if (!ok) break;
#pragma unroll
                for (int t = 0; t < F::kQTiles; ++t) issue_scores<D, kHalf>(tmem, k_desc0 + F::kDescStageK * j, t, j, &s.s_full[t][j]);
            }
            for (int j = 0; j < tiles && ok; ++j) {
                const int stage = j % kStages, buffer = j & 1;
                const bool more = j + 2 < tiles;
                const int next_stage = (j + 2) % kStages;
                bool next_ready = !more;
                bool served[F::kQTiles] = {};
                const long long start_clock = clock64();
                // Statistics: p_full(j) only tells that buffer j may take S(j + 2); for the last two
                // tiles there is nothing to issue, so they are not waited for. (Waiting would be wrong:
                // a softmax warp releases tile j after S(j + 1) is issued -- which keeps it at most one
                // phase ahead -- but the last tile has no S(j + 1), so its release may complete a second
                // p_full phase before this warp has seen the first, and a parity wait cannot tell two
                // completed phases from none.)
                int remaining = kStats && !more ? 0 : F::kQTiles;
                while (remaining > 0 && ok) {
#pragma unroll
                    for (int t = 0; t < F::kQTiles; ++t) {
                        if (!ok || served[t] || !mbar_test_wait_warp(&s.p_full[t], j & 1)) continue;
                        if (lane == 0) RK_TRACE(j, t);
                        tc_fence_after();
                        if constexpr (!kStats)
                            issue_values<D, kHalf>(tmem, v_desc0 + F::kDescStageV * stage, t, buffer, &s.pv_done[t]);
                        if (more) {
                            if (!next_ready) {
                                next_ready = mbar_wait_warp(&s.kv_ready[next_stage], ((j + 2) / kStages) & 1);
                                if (!next_ready) {
                                    ok = false;
                                    continue;
                                }
                                tc_fence_after();
                            }
                            issue_scores<D, kHalf>(tmem, k_desc0 + F::kDescStageK * next_stage, t, buffer, &s.s_full[t][buffer]);
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
    } else if (!kPrepared && warp >= F::kSplitWarp) {
        // ---------------------------------------------------------------- FP16 split
        // Split warp w owns key rows [32w, 32w + 32) of every tile; its ballot is their mask.
        // K: lane = one key row -> its row-layout chunks [k0 | k1]. V: item = (key group of 8 rows,
        // chunk of 4 features) -> the 4 features' 8-key FP16 chunks of v0^T and v1^T.
        const int w = warp - F::kSplitWarp;
        const unsigned char *mask = p.mask + static_cast<long long>(b) * p.keys;
        const int row = 32 * w + lane;  // K row of this lane
        // The prefetched tiles are converted without waiting for the visible-tile count (which
        // comes from a mask read); tiles of them past the last visible key are converted for
        // nothing and never consumed.
        int tiles = prefetched;
        bool counted = false;
        for (int j = 0; j < tiles || !counted; ++j) {
            if (!counted && j >= prefetched) {
                tiles = __shfl_sync(0xffffffffu, visible_tiles(), 0);
                counted = true;
                if (j >= tiles) break;
            }
            const int stage = j % kStages, use = j / kStages;
            if constexpr (kHalf) {
                // FP16 storage: the MMAs read K from the TMA tile; V is transposed, masked rows zeroed.
                if (!__all_sync(0xffffffffu, mbar_wait(&s.kv_full[stage], use & 1))) break;
                const int key = first + j * kKeyTile + row;
                const uint32_t bits = __ballot_sync(0xffffffffu, key < last && mask[key] != 0);
                if (lane == 0) s.header[stage].mask[w] = bits;
                transpose_values<D>(s.v_raw[stage], s.vt16[stage], w, lane, bits);
                fence_proxy_async_shared();
                mbar_arrive(&s.kv_ready[stage]);
                continue;
            } else {
            // Both split warps pass the named barrier below before either may give up, so a
            // failed wait can never leave one of them blocked in bar.sync.
            const bool landed = __all_sync(0xffffffffu, mbar_wait(&s.kv_full[stage], use & 1));
            if (lane == 0) RK_TRACE(j, 13 + w);
            const int key = first + j * kKeyTile + row;
            const uint32_t bits = __ballot_sync(0xffffffffu, key < last && mask[key] != 0);
            const bool keep_row = (bits >> lane) & 1;
            // This lane's K row and V items stay in registers from the max pass to the conversion.
            // V item (group, fchunk) covers rows 8 group .. 8 group + 7, all rows of this warp.
            float4 kx[D / 4], vx[D / 32][8];
            float kmax = 0.f, vmax = 0.f;
#pragma unroll
            for (int c = 0; c < D / 4; ++c) {
                kx[c] = raw_chunk<D>(s.k_raw[stage], row, c);
                if (!keep_row) kx[c] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
            if constexpr (kRotary && !kPrepared) {
                if (keep_row) {
                    float4 cs[8], sn[8];
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        cs[c] = raw_chunk<32>(s.cos_raw[stage], row, c);
                        sn[c] = raw_chunk<32>(s.sin_raw[stage], row, c);
                    }
                    rotate_row32(kx, cs, sn);
                }
            }
#pragma unroll
            for (int c = 0; c < D / 4; ++c)
                kmax = max3(kmax, fmaxf(fabsf(kx[c].x), fabsf(kx[c].y)), fmaxf(fabsf(kx[c].z), fabsf(kx[c].w)));
#pragma unroll
            for (int item = 0; item < (kStats ? 0 : D / 32); ++item) {  // statistics: no V
                const int index = 64 * item + row;  // 0 .. 2D - 1
                const int group = index >> 3 & 7, fchunk = (index & 7) + 8 * (index >> 6);
#pragma unroll
                for (int r = 0; r < 8; ++r) {
                    const int vrow = 8 * group + r;
                    vx[item][r] = raw_chunk<D>(s.v_raw[stage], vrow, fchunk);
                    if (!((bits >> (vrow & 31)) & 1)) vx[item][r] = make_float4(0.f, 0.f, 0.f, 0.f);
                    vmax = max3(vmax, fmaxf(fabsf(vx[item][r].x), fabsf(vx[item][r].y)),
                                fmaxf(fabsf(vx[item][r].z), fabsf(vx[item][r].w)));
                }
            }
            // Everything of the raw stage is in registers now: the producer may refill it.
            if constexpr (F::kEarlyRawRefill) mbar_arrive(&s.raw_free[stage]);
#pragma unroll
            for (int offset = 16; offset; offset >>= 1) {
                kmax = fmaxf(kmax, __shfl_xor_sync(0xffffffffu, kmax, offset));
                vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, offset));
            }
            // The converted stage (and the stage's mask and exponents, which the softmax threads
            // read for tile j - kStages) is rewritten only after the MMAs of that tile finished.
            const bool stage_free = !F::kEarlyRawRefill || j < kStages ||
                                    __all_sync(0xffffffffu, mbar_wait(&s.kv_empty[stage], ((j / kStages) - 1) & 1));
            if (lane == 0) {
                s.split_max[w][0] = kmax;
                s.split_max[w][1] = vmax;
                s.split_ok[w] = landed && stage_free;
                s.header[stage].mask[w] = bits;
            }
            asm volatile("bar.sync 1, 64;" ::: "memory");
            if (!(s.split_ok[0] && s.split_ok[1])) break;
            const int k_exponent = fp16_scale_exponent(fmaxf(s.split_max[0][0], s.split_max[1][0]));
            const int v_exponent = fp16_scale_exponent(fmaxf(s.split_max[0][1], s.split_max[1][1]));
            asm volatile("bar.sync 1, 64;" ::: "memory");  // split_max is rewritten for the next tile
            if (threadIdx.x == F::kSplitWarp * 32) {
                s.header[stage].k_exponent = k_exponent;
                s.header[stage].v_exponent = v_exponent;
            }
            const float k_scale = exp2_int(k_exponent), v_scale = exp2_int(v_exponent);
            // K row: features 8m..8m+7 -> k0 chunk m and k1 chunk m of the row layout
#pragma unroll
            for (int m = 0; m < D / 8; ++m) {
                const float x[8] = {kx[2 * m].x, kx[2 * m].y, kx[2 * m].z, kx[2 * m].w,
                                    kx[2 * m + 1].x, kx[2 * m + 1].y, kx[2 * m + 1].z, kx[2 * m + 1].w};
                uint4 c0, c1;
                split_pack8<false>(x, k_scale, c0, c1);
                *row_chunk<D>(s.k16[stage], row, 0, m) = c0;
                *row_chunk<D>(s.k16[stage], row, 1, m) = c1;
            }
            // V^T rows f (v0) and D + f (v1), keys 8g..8g+7 = 16-byte chunk g (swizzled by f % 8)
            uint4 *vt16 = reinterpret_cast<uint4 *>(s.vt16[stage]);
#pragma unroll
            for (int item = 0; item < (kStats ? 0 : D / 32); ++item) {
                const int index = 64 * item + row;
                const int group = index >> 3 & 7, fchunk = (index & 7) + 8 * (index >> 6);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int f = 4 * fchunk + e;
                    float column[8];
#pragma unroll
                    for (int r = 0; r < 8; ++r) {
                        const float4 &x = vx[item][r];
                        column[r] = e == 0 ? x.x : e == 1 ? x.y : e == 2 ? x.z : x.w;
                    }
                    uint4 c0, c1;
                    split_pack8<false>(column, v_scale, c0, c1);
                    vt16[f * 8 + (group ^ (f & 7))] = c0;
                    vt16[(D + f) * 8 + (group ^ (f & 7))] = c1;
                }
            }
            fence_proxy_async_shared();
            if (lane == 0) RK_TRACE(j, w == 0 ? 3 : 15);
            mbar_arrive(&s.kv_ready[stage]);
            }
        }
    } else {
        // ---------------------------------------------------------------- softmax / epilogue
        const int tile = kRowThreads == 2 ? 0 : warp >> 2;  // Q tile (0 = A, 1 = B)
        const int part = kRowThreads == 2 ? warp >> 2 : 0;  // two threads per row: this thread's half
        const int row_in_tile = threadIdx.x & (kQTile - 1);
        // query and row_valid: this thread's row, computed with the Q prefetch above
        const uint32_t lane_base = tmem_lane_address(tmem, warp) + tile * F::kColTile;
        const bool tracer = row_in_tile == 0;

        int q_exponent = 0;
        if constexpr (kHalf) {  // Q row as FP16 pairs in TMEM, unscaled
            float packed[D / 2];
#pragma unroll
            for (int c = 0; c < D / 8; ++c) {
                const uint4 v = q_chunks[c];
                packed[4 * c] = __uint_as_float(v.x);
                packed[4 * c + 1] = __uint_as_float(v.y);
                packed[4 * c + 2] = __uint_as_float(v.z);
                packed[4 * c + 3] = __uint_as_float(v.w);
            }
#pragma unroll
            for (int c = 0; c < D / 2; c += 16) {
                if constexpr (D == 16)
                    tmem_store8_async(lane_base + F::kColQ0, packed);
                else
                    tmem_store8x2_async(lane_base + F::kColQ0 + c, packed + c, lane_base + F::kColQ0 + c + 8, packed + c + 8);
            }
            tmem_wait_store();
            tc_fence_before();
            mbar_arrive(&s.q_ready);
        } else {  // Q row -> scaled by 1/sqrt(D) and 2^q_exponent, split into FP16 q0/q1 pairs in TMEM
            float x[D];
            float4 raw[D / 4];
#pragma unroll
            for (int c = 0; c < D / 4; ++c)
                raw[c] = make_float4(__uint_as_float(q_chunks[c].x), __uint_as_float(q_chunks[c].y),
                                     __uint_as_float(q_chunks[c].z), __uint_as_float(q_chunks[c].w));
            if constexpr (kRotary) {
                if (row_valid) rotate_row32(raw, q_cos, q_sin);
            }
            float qmax = 0.f;
#pragma unroll
            for (int c = 0; c < D / 4; ++c) {
                x[4 * c] = raw[c].x * p.scale;
                x[4 * c + 1] = raw[c].y * p.scale;
                x[4 * c + 2] = raw[c].z * p.scale;
                x[4 * c + 3] = raw[c].w * p.scale;
#pragma unroll
                for (int e = 0; e < 4; ++e) qmax = fmaxf(qmax, fabsf(x[4 * c + e]));
            }
            q_exponent = fp16_scale_exponent(qmax);
            const float q_scale = exp2_int(q_exponent);
#pragma unroll
            for (int half = 0; half < D / 32; ++half) {
                float packed0[16], packed1[16];
#pragma unroll
                for (int c = 0; c < 16; ++c) {
                    uint32_t p0, p1;
                    split_pack2<false>(x[32 * half + 2 * c], x[32 * half + 2 * c + 1], q_scale, p0, p1);
                    packed0[c] = __uint_as_float(p0);
                    packed1[c] = __uint_as_float(p1);
                }
                if constexpr (kRowThreads == 2) {  // each of the row's two threads stores half the pairs
                    if (part == 0)
                        tmem_store8x2_async(lane_base + F::kColQ0, packed0, lane_base + F::kColQ1, packed1);
                    else
                        tmem_store8x2_async(lane_base + F::kColQ0 + 8, packed0 + 8, lane_base + F::kColQ1 + 8, packed1 + 8);
                    tmem_wait_store();
                } else {
                    tmem_store16x2(lane_base + F::kColQ0 + 16 * half, packed0, lane_base + F::kColQ1 + 16 * half, packed1);
                }
            }
            tc_fence_before();
            mbar_arrive(&s.q_ready);
        }

        if constexpr (kRowThreads == 2) {
            // Two threads per row: this thread takes keys 32 part .. 32 part + 31 of every tile and
            // output columns 16 part .. 16 part + 15. The row's two threads (warps w and w + 4, the
            // same TMEM lanes) exchange their partial row max each tile through shared memory and
            // keep the same row max, sum and exponent (both read the row-sum column).
            const int quarter = warp & 3;
            float row_max = -INFINITY, row_sum = 0.f;  // row_sum carries the 2^14 of P
            float o[16];                               // this thread's output columns, scaled by 2^o_exp
#pragma unroll
            for (int c = 0; c < 16; ++c) o[c] = 0.f;
            int o_exp = kNoExponent;
            float pending_weight = 0.f;
            int pending_exponent = 0;
            bool ok = true;
            const int tiles = __shfl_sync(0xffffffffu, visible_tiles(), 0);
            for (int j = 0; j < tiles && ok; ++j) {
                const int stage = j % kStages, use = j / kStages, buffer = j & 1;
                const uint32_t pbuf = lane_base + F::kColBuffer + buffer * F::kBufferColumns;
                ok = __all_sync(0xffffffffu, mbar_wait(&s.s_full[0][buffer], (j >> 1) & 1) && mbar_wait(&s.kv_full[stage], use & 1));
                if (!ok) break;
                if (tracer && part == 0) RK_TRACE(j, 4);
                tc_fence_after();
                float sc[32];
                tmem_load32(pbuf + 32 * part, sc);
                const int k0 = first + j * kKeyTile + 32 * part;
                uint32_t active = row_valid ? s.header[stage].mask[part] : 0u;
                if (p.radius >= 0) {
                    const int lo_col = max(0, query - p.radius - k0), hi_col = min(31, query + p.radius - k0);
                    active &= lo_col > hi_col ? 0u : ((~0u) >> (31 - (hi_col - lo_col))) << lo_col;
                }
                const float s_scale = exp2_int(-(q_exponent + s.header[stage].k_exponent));
                const int v_exponent = s.header[stage].v_exponent;
                if (active != ~0u) {
#pragma unroll
                    for (int c = 0; c < 32; ++c) sc[c] = (active >> c) & 1 ? sc[c] : -INFINITY;
                }
                float partial_max[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
                for (int c = 0; c < 32; c += 2) partial_max[(c >> 1) & 3] = max3(partial_max[(c >> 1) & 3], sc[c], sc[c + 1]);
                const float half_max = max3(partial_max[0], partial_max[1], fmaxf(partial_max[2], partial_max[3]));
                // The other half's maximum: written for tile parity j & 1, read after both threads of
                // the quarter arrived (a thread rewrites this slot only two tiles later, after the
                // next meeting, which needs the partner's arrival after its read).
                s.row_exchange[j & 1][part][row_in_tile] = half_max;
                mbar_arrive(&s.pair_bar[quarter]);
                ok = __all_sync(0xffffffffu, mbar_wait(&s.pair_bar[quarter], j & 1));
                if (!ok) break;
                const float raw_max = fmaxf(half_max, s.row_exchange[j & 1][part ^ 1][row_in_tile]);
                const float tile_max = raw_max == -INFINITY ? -INFINITY : raw_max * s_scale;
                if (tracer && part == 0) RK_TRACE(j, 5);
                const float next = fmaxf(row_max, tile_max);
                const float old_weight = isfinite(row_max) ? fast_exp2((row_max - next) * kLog2e) : 0.f;
                const float slope = s_scale * kLog2e;
                const float offset = fmaf(-next, kLog2e, 14.f);  // P' = 2^14 exp(S - max) = exp2(S * slope + offset)
                // P(j) may be written before Ot(j - 1) is folded: only the p_full arrival below lets
                // the MMA warp start P(j).V, which overwrites Ot.
                const uint32_t pcols = pbuf + 16 * part;
                if (__all_sync(0xffffffffu, isfinite(offset) && slope > 0.f))
                    exp_split_store<true, false, true, 32>(sc, slope, offset, pcols);
                else
                    exp_split_store<false, false, true, 32>(sc, slope, offset, pcols);
                if (j > 0) {  // fold tile j-1 before P(j).V overwrites its Ot
                    ok = __all_sync(0xffffffffu, mbar_wait(&s.pv_done[0], (j - 1) & 1));
                    if (!ok) {
                        tmem_wait_store();  // no store may be in flight when TMEM is released
                        break;
                    }
                    tc_fence_after();
                    float ot[16], sum;
                    tmem_load16_1(lane_base + F::kColO + 16 * part, ot, lane_base + F::kColSum, sum);
                    fold_prepared<16>(o, row_sum, o_exp, ot, sum, pending_weight, pending_exponent);
                }
                tmem_wait_store();
                tc_fence_before();
                if (tracer && part == 0) RK_TRACE(j, 6);
                mbar_arrive(&s.p_full[0]);
                row_max = next;
                pending_weight = old_weight;
                pending_exponent = v_exponent;
            }
            // Epilogue (AttentionFlash32.h:157-169): O / total; fully masked rows give 0 and {-inf, 0}.
            if (tiles > 0 && ok) {
                ok = __all_sync(0xffffffffu, mbar_wait(&s.pv_done[0], (tiles - 1) & 1));
                tc_fence_after();
                if (ok) {
                    float ot[16], sum;
                    tmem_load16_1(lane_base + F::kColO + 16 * part, ot, lane_base + F::kColSum, sum);
                    fold_prepared<16>(o, row_sum, o_exp, ot, sum, pending_weight, pending_exponent);
                }
            }
            if (row_valid) {
                const float total = ok ? row_sum : NAN;
                const bool nan_out = isnan(total) && !p.zero_nan_rows;
                const float out_scale = exp2_int(-o_exp) / total;
#pragma unroll
                for (int c = 0; c < 16; ++c) o[c] = total > 0.f ? o[c] * out_scale : nan_out ? NAN : 0.f;
                float *out = p.o.row(b, h, query) + 16 * part;
                if (args.vec_out) {
#pragma unroll
                    for (int c = 0; c < 4; ++c)
                        reinterpret_cast<float4 *>(out)[c] = make_float4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
                } else {
#pragma unroll
                    for (int c = 0; c < 16; ++c) out[c] = o[c];
                }
                if (part == 0) {
                    const long long row = (static_cast<long long>(b) * p.heads + h) * p.queries + query;
                    p.lse[row * 2] = total > 0.f ? row_max : nan_out ? NAN : -INFINITY;
                    p.lse[row * 2 + 1] = total > 0.f ? total * (1.f / kPScale) : nan_out ? NAN : 0.f;
                }
            }
        } else {
            float row_max = -INFINITY, row_sum = 0.f;  // row_sum carries the 2^14 of P
            float o[D];                                // running output, scaled by 2^o_exp
    #pragma unroll
            for (int c = 0; c < D; ++c) o[c] = 0.f;
            int o_exp = kNoExponent;
            float pending_weight = 0.f;  // exp(m_(j-2) - m_(j-1)), applied when tile j-1 is folded
            int pending_exponent = 0;    // c_(j-1): the V exponent of tile j-1
            bool ok = true;
            const int tiles = __shfl_sync(0xffffffffu, visible_tiles(), 0);
            for (int j = 0; j < tiles && ok; ++j) {
                const int stage = j % kStages, use = j / kStages, buffer = j & 1;
                const uint32_t pbuf = lane_base + F::kColBuffer + buffer * F::kBufferColumns;
                // The stage's header: converted by the split warps (kv_ready), or landed with the
                // prepared image (kv_full).
                ok = __all_sync(0xffffffffu, mbar_wait(&s.s_full[tile][buffer], (j >> 1) & 1) &&
                                                     mbar_wait(kPrepared ? &s.kv_full[stage] : &s.kv_ready[stage], use & 1));
                if (!ok) break;
                tc_fence_after();
                float sc[64];
                tmem_load64(pbuf, sc);
                if (tracer) RK_TRACE(j, 4 + 4 * tile);
                RK_WARP_TRACE(j, 0);
                // Visible keys of this row in the tile: key mask x radius window x valid row.
                const int k0 = first + j * kKeyTile;
                uint64_t active = row_valid ? (static_cast<uint64_t>(s.header[stage].mask[0]) |
                                               (static_cast<uint64_t>(s.header[stage].mask[1]) << 32))
                                            : 0ull;
                if (p.radius >= 0) {
                    const int lo_col = max(0, query - p.radius - k0), hi_col = min(kKeyTile - 1, query + p.radius - k0);
                    active &= lo_col > hi_col ? 0ull : ((~0ull) >> (63 - (hi_col - lo_col))) << lo_col;
                }
                // TMEM S -> scaled score (FP16 storage: S is the plain dot product)
                const float s_scale = kHalf ? p.scale : exp2_int(-(q_exponent + s.header[stage].k_exponent));
                const int v_exponent = kHalf ? 0 : s.header[stage].v_exponent;
                if constexpr (kStats) {
                    // S and the stage's mask and exponent are in registers: S(j + 2) may overwrite the
                    // buffer and the stage may be refilled. The MMA warp must have seen this tile's
                    // release of buffer j - 1 before this arrival (two arrivals it has not seen would
                    // complete two phases of p_full, which its parity wait cannot tell from none); it
                    // issues S(j + 1) only after seeing that release, so wait for S(j + 1) first.
                    if (j + 1 < tiles)
                        ok = __all_sync(0xffffffffu, mbar_wait(&s.s_full[tile][buffer ^ 1], ((j + 1) >> 1) & 1));
                    if (!ok) break;
                    tc_fence_before();
                    mbar_arrive(&s.p_full[tile]);
                }
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
                if constexpr (kStats) {
                    // Statistics only: the row sum of P' in FP32, no P, no output.
                    float partial[4] = {0.f, 0.f, 0.f, 0.f};
    #pragma unroll
                    for (int c = 0; c < 64; ++c)
                        partial[c & 3] += sc[c] == -INFINITY ? 0.f : fast_exp2(fmaf(sc[c], slope, offset));
                    row_sum = fmaf(row_sum, old_weight, (partial[0] + partial[1]) + (partial[2] + partial[3]));
                    row_max = next;
                    continue;
                }
                // P(j) may be written before Ot(j - 1) is folded: only the p_full arrival below lets
                // the MMA warp start P(j).V, which overwrites Ot. The TMEM stores inside are
                // warp-collective, so the branch is taken by the whole warp (the explicit path is
                // exact for finite rows too).
                constexpr bool kPackedSplit = kHalf || D == 64 || F::kQTiles == 1;
                RK_WARP_TRACE(j, 5);
                const float tile_sum = __all_sync(0xffffffffu, isfinite(offset) && slope > 0.f)
                                               ? exp_split_store<true, kHalf, kPackedSplit>(sc, slope, offset, pbuf)
                                               : exp_split_store<false, kHalf, kPackedSplit>(sc, slope, offset, pbuf);
                if constexpr (kHalf) row_sum = fmaf(row_sum, old_weight, tile_sum);  // kept in units of the new max
                RK_WARP_TRACE(j, 2);
                if constexpr (kPrepared) {
                    if (j > 0) {  // fold tile j-1 before P(j).V overwrites its Ot
                        ok = __all_sync(0xffffffffu, mbar_wait(&s.pv_done[tile], (j - 1) & 1));
                        if (!ok) {
                            tmem_wait_store();  // no store may be in flight when TMEM is released
                            break;
                        }
                        tc_fence_after();
                        float ot[32], sum;
                        tmem_load32_1(lane_base + F::kColO, ot, lane_base + F::kColSum, sum);
                        fold_prepared(o, row_sum, o_exp, ot, sum, pending_weight, pending_exponent);
                    }
                } else if (j > 0) {  // fold tile j-1 before P(j).V overwrites its Ot
                    ok = __all_sync(0xffffffffu, mbar_wait(&s.pv_done[tile], (j - 1) & 1));
                    if (!ok) {
                        tmem_wait_store();  // no store may be in flight when TMEM is released
                        break;
                    }
                    tc_fence_after();
                    fold_output<D, kHalf>(o, row_sum, o_exp, lane_base, pending_weight, pending_exponent);
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
            if (!kStats && tiles > 0 && ok) {
                ok = __all_sync(0xffffffffu, mbar_wait(&s.pv_done[tile], (tiles - 1) & 1));
                tc_fence_after();
                if (ok) {
                    if constexpr (kPrepared) {
                        float ot[32], sum;
                        tmem_load32_1(lane_base + F::kColO, ot, lane_base + F::kColSum, sum);
                        fold_prepared(o, row_sum, o_exp, ot, sum, pending_weight, pending_exponent);
                    } else {
                        fold_output<D, kHalf>(o, row_sum, o_exp, lane_base, pending_weight, pending_exponent);
                    }
                }
            }
            if (row_valid) {
                const float total = ok ? row_sum : NAN;
                const bool nan_out = isnan(total) && !p.zero_nan_rows;
                const float out_scale = exp2_int(-o_exp) / total;
    #pragma unroll
                for (int c = 0; c < D; ++c) o[c] = total > 0.f ? o[c] * out_scale : nan_out ? NAN : 0.f;
                if constexpr (kHalf) {
                    __half *out = p.o.row_as<__half>(b, h, query);
                    if (args.vec_out) {
    #pragma unroll
                        for (int c = 0; c < D / 8; ++c)
                            reinterpret_cast<uint4 *>(out)[c] =
                                    make_uint4(pack_half2(o[8 * c], o[8 * c + 1]), pack_half2(o[8 * c + 2], o[8 * c + 3]),
                                               pack_half2(o[8 * c + 4], o[8 * c + 5]), pack_half2(o[8 * c + 6], o[8 * c + 7]));
                    } else {
    #pragma unroll
                        for (int c = 0; c < D; ++c) out[c] = __float2half_rn(o[c]);
                    }
                } else if constexpr (!kStats) {  // statistics: no output rows
                    float *out = p.o.row(b, h, query);
                    if (args.vec_out) {
    #pragma unroll
                        for (int c = 0; c < kWidth / 4; ++c)
                            reinterpret_cast<float4 *>(out)[c] = make_float4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
                    } else {
    #pragma unroll
                        for (int c = 0; c < kWidth; ++c) out[c] = o[c];
                    }
                }
                const long long row = (static_cast<long long>(b) * p.heads + h) * p.queries + query;
                p.lse[row * 2] = total > 0.f ? row_max : nan_out ? NAN : -INFINITY;
                p.lse[row * 2 + 1] = total > 0.f ? total * (1.f / kPScale) : nan_out ? NAN : 0.f;
            }
        }
    }

    RK_CTA_TRACE(2);
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, F::kTmemColumns);
    }
    RK_CTA_TRACE(3);
}

// Operand pre-pass of the prepared d = 32 forward: one CTA of 256 threads per 64-key tile of one
// (batch, head). It builds the tile's stage image as the forward's split warps build it in shared
// memory -- keys that are masked or past the sequence zeroed with their mask bits clear; K and V
// scaled by the powers of two that bring the tile's largest magnitudes into [2^14, 2^15) and split
// into FP16 pairs (x0 rounded to nearest, x1 the rounded residual); K as [k0 | k1] rows, V as
// v1^T / v0^T rows, 128B-swizzled -- and the tile's header. Each head's K and V are thus read and
// split once, instead of once per query block.
// Thread = (key row = thread / 4, features 8q .. 8q + 7 with q = thread % 4): warp g holds key rows
// 8g .. 8g + 7, so the V^T chunk of feature f and key group g (V[8g .. 8g + 7][f]) is gathered by
// an 8 x 8 register transpose among the warp's lanes with the same q.
// kRotary: each K row is first rotated by its token's tables (rotate_pair, as rotate_row32 does in
// the forward's split warps): features f and f + 16 sit in lanes q and q ^ 2 of the same row.
constexpr int kPrepareThreads = 256;

template <bool kRotary>
__global__ void __launch_bounds__(kPrepareThreads) prepare_kv_kernel(const AttentionParams p, uint8_t *images, StageHeader *headers,
                                                                     int tiles_per_head) {
    grid_launch_dependents();  // the forward may be scheduled now; it waits for this grid to complete
    __shared__ float warp_max[2][kPrepareThreads / 32];
    __shared__ uint32_t mask_bits[2];
    const long long tile = blockIdx.x;
    const int t = static_cast<int>(tile % tiles_per_head);
    const int bh = static_cast<int>(tile / tiles_per_head);
    const int h = bh % p.heads, b = bh / p.heads;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const unsigned char *mask = p.mask + static_cast<long long>(b) * p.keys;
    const int row = threadIdx.x >> 2, q = threadIdx.x & 3;
    const int key = t * kKeyTile + row;
    // The rows are read whether or not the mask shows the key (past the sequence: row 0), so that
    // the loads do not wait for the mask byte; masked rows are zeroed afterwards.
    const bool in_range = key < p.keys;
    const int read_key = in_range ? key : 0;
    const unsigned char key_byte = in_range ? mask[key] : 0;
    const float4 *krow = reinterpret_cast<const float4 *>(p.k.row(b, h, read_key)) + 2 * q;
    const float4 *vrow = reinterpret_cast<const float4 *>(p.v.row(b, h, read_key)) + 2 * q;
    const float4 k0 = __ldg(krow), k1 = __ldg(krow + 1), v0 = __ldg(vrow), v1 = __ldg(vrow + 1);
    float kx[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
    float vx[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    if constexpr (kRotary) {
        const float4 *c4 = reinterpret_cast<const float4 *>(p.cos_row(b, read_key)) + 2 * q;
        const float4 *s4 = reinterpret_cast<const float4 *>(p.sin_row(b, read_key)) + 2 * q;
        const float4 c0 = __ldg(c4), c1 = __ldg(c4 + 1), s0 = __ldg(s4), s1 = __ldg(s4 + 1);
        const float cs[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
        const float sn[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
        const bool low = q < 2;  // features 8q.. are the low halves f of the pairs (f, f + 16)
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const float partner = __shfl_xor_sync(0xffffffffu, kx[e], 2);
            float out_lo, out_hi;
            if (low)
                rotate_pair<false>(kx[e], partner, cs[e], cs[e], sn[e], sn[e], out_lo, out_hi);
            else
                rotate_pair<false>(partner, kx[e], cs[e], cs[e], sn[e], sn[e], out_lo, out_hi);
            kx[e] = low ? out_lo : out_hi;
        }
    }
    const bool visible = in_range && key_byte != 0;
    float kmax = 0.f, vmax = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        kx[e] = visible ? kx[e] : 0.f;
        vx[e] = visible ? vx[e] : 0.f;
        kmax = fmaxf(kmax, fabsf(kx[e]));
        vmax = fmaxf(vmax, fabsf(vx[e]));
    }
#pragma unroll
    for (int offset = 16; offset; offset >>= 1) {
        kmax = fmaxf(kmax, __shfl_xor_sync(0xffffffffu, kmax, offset));
        vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, offset));
    }
    if (lane == 0) {
        warp_max[0][warp] = kmax;
        warp_max[1][warp] = vmax;
    }
    if (warp < 2) {  // the tile's visible keys, 32 per warp
        const int mkey = t * kKeyTile + threadIdx.x;
        const uint32_t bits = __ballot_sync(0xffffffffu, mkey < p.keys && mask[mkey] != 0);
        if (lane == 0) mask_bits[warp] = bits;
    }
    // V^T chunk of feature 8q + lane / 4 and key group `warp`: transpose the 8 x 8 block
    // (row = lane / 4, element e) among the lanes with this q, three swap stages on lane bits 2-4.
    const int r_local = lane >> 2;
#pragma unroll
    for (int m = 1; m < 8; m <<= 1) {
        const bool upper = (r_local & m) != 0;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            if (e & m) continue;
            const float send = upper ? vx[e] : vx[e | m];
            const float received = __shfl_xor_sync(0xffffffffu, send, 4 * m);
            if (upper)
                vx[e] = received;
            else
                vx[e | m] = received;
        }
    }
    __syncthreads();
    float kmax_tile = warp_max[0][0], vmax_tile = warp_max[1][0];
#pragma unroll
    for (int w = 1; w < kPrepareThreads / 32; ++w) {
        kmax_tile = fmaxf(kmax_tile, warp_max[0][w]);
        vmax_tile = fmaxf(vmax_tile, warp_max[1][w]);
    }
    const int k_exponent = fp16_scale_exponent(kmax_tile), v_exponent = fp16_scale_exponent(vmax_tile);
    uint8_t *image = images + tile * kImageBytes;
    uint4 c0, c1;
    // K row: features 8q..8q+7 -> chunk q of k0 and of k1 in the row layout
    split_pack8<true>(kx, exp2_int(k_exponent), c0, c1);
    uint32_t *k16 = reinterpret_cast<uint32_t *>(image);
    *row_chunk<32>(k16, row, 0, q) = c0;
    *row_chunk<32>(k16, row, 1, q) = c1;
    // V^T rows f (v1) and 32 + f (v0), the order issue_values_prepared reads them in; the 16-byte
    // chunk of key group g sits at position g ^ (f % 8) of its row.
    const int f = 8 * q + r_local, position = warp ^ (f & 7);
    split_pack8<true>(vx, exp2_int(v_exponent), c0, c1);
    uint4 *vt16 = reinterpret_cast<uint4 *>(image + kImageKBytes);
    vt16[(32 + f) * 8 + position] = c0;
    vt16[f * 8 + position] = c1;
    if (threadIdx.x == 0) {
        StageHeader header;
        header.mask[0] = mask_bits[0];
        header.mask[1] = mask_bits[1];
        header.k_exponent = k_exponent;
        header.v_exponent = v_exponent;
        headers[tile] = header;
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

// [batch][heads][tokens][width] with the given element strides, FP32 (box = 32 features x 64
// tokens) or FP16 (box = 64 features x 64 tokens; for width < 64 the features past the width
// are the TMA's zero fill). 128-byte box rows, 128B swizzle.
bool make_tensor_map(CUtensorMap *map, const Tensor &t, int width, int batch, int heads, int tokens, bool half) {
    auto encode = encode_function();
    if (encode == nullptr) return false;
    const cuuint64_t element = half ? 2 : 4;
    const cuuint64_t dims[4] = {static_cast<cuuint64_t>(width), static_cast<cuuint64_t>(tokens), static_cast<cuuint64_t>(heads),
                                static_cast<cuuint64_t>(batch)};
    const cuuint64_t strides[3] = {static_cast<cuuint64_t>(t.st) * element, static_cast<cuuint64_t>(t.sh) * element,
                                   static_cast<cuuint64_t>(t.sb) * element};
    const cuuint32_t box[4] = {half ? 64u : 32u, static_cast<cuuint32_t>(kKeyTile), 1, 1};
    const cuuint32_t element_strides[4] = {1, 1, 1, 1};
    return encode(map, half ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float *>(t.data), dims,
                  strides, box, element_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Strides that TMA accepts (positive multiples of 16 bytes below 2^40 bytes) and a 16-byte aligned
// base; `per16` = elements per 16 bytes.
bool positive_tma_strides(const Tensor &t, int per16) {
    const long long limit = 1ll << 38;
    return t.st > 0 && t.sh > 0 && t.sb > 0 && t.st % per16 == 0 && t.sh % per16 == 0 && t.sb % per16 == 0 && t.st < limit &&
           t.sh < limit && t.sb < limit && (reinterpret_cast<uintptr_t>(t.data) & 15u) == 0;
}

template <int D, bool kHalf, bool kRotary = false, int kTiles = Forward<D, kHalf>::kQTiles>
constexpr int shared_bytes() {
    if constexpr (kRotary)
        return static_cast<int>(sizeof(RotaryStorage<D, kTiles>)) + 1024;
    else
        return static_cast<int>(sizeof(SharedStorage<D, kHalf, kTiles>)) + 1024;
}
template <int D, bool kHalf, int kTiles = Forward<D, kHalf>::kQTiles>
constexpr bool layout_ok() {
    using F = Forward<D, kHalf, kTiles>;
    using S = SharedStorage<D, kHalf, kTiles>;
    return (kHalf || sizeof(S::k16[0]) == 64 * 2 * D * 2) && sizeof(S::vt16[0]) == F::kVRows * 128 &&
           sizeof(S::vt16[0]) % 1024 == 0 && sizeof(S::k_raw[0]) % 1024 == 0 &&
           F::kColSum + (kHalf ? 0 : 16) <= (F::kQTiles == 2 ? F::kColTile : F::kTmemColumns) &&
           shared_bytes<D, kHalf, false, kTiles>() <= 227 * 1024;
}
static_assert(layout_ok<32, false>() && layout_ok<32, false, 1>() && layout_ok<64, false>() && layout_ok<16, true>() &&
                      layout_ok<32, true>() && layout_ok<64, true>(),
              "operand tiles, TMEM columns and shared memory budget");
static_assert(shared_bytes<32, false, true>() <= 227 * 1024 && shared_bytes<32, false, true, 1>() <= 227 * 1024,
              "rotary tables fit beside the d = 32 stages");

// Rotary table [batch][rows][32] FP32 (token stride st, batch stride sb, 0 = one table for every
// sequence) as a 4-D map {32, rows, 1, batch} with the K boxes' shape: box = 32 features x 64 rows.
bool make_table_map(CUtensorMap *map, const float *table, long long sb, long long st, int rows, int batch) {
    auto encode = encode_function();
    if (encode == nullptr || st <= 0 || sb < 0) return false;
    const cuuint64_t dims[4] = {32, static_cast<cuuint64_t>(rows), 1, static_cast<cuuint64_t>(sb > 0 ? batch : 1)};
    const cuuint64_t row_bytes = static_cast<cuuint64_t>(st) * 4;
    const cuuint64_t strides[3] = {row_bytes, row_bytes * static_cast<cuuint64_t>(rows),
                                   sb > 0 ? static_cast<cuuint64_t>(sb) * 4 : row_bytes * static_cast<cuuint64_t>(rows)};
    const cuuint32_t box[4] = {32, static_cast<cuuint32_t>(kKeyTile), 1, 1};
    const cuuint32_t element_strides[4] = {1, 1, 1, 1};
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float *>(table), dims, strides, box, element_strides,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int D, bool kHalf, int kWidth = D, bool kRotary = false, int kTiles = Forward<D, kHalf>::kQTiles,
          bool kStats = false, bool kChained = false>
int launch_tiles(const AttentionParams &p, cudaStream_t stream) {
    using F = Forward<D, kHalf, kTiles>;
    CUtensorMap tmap_k, tmap_v;
    if (!make_tensor_map(&tmap_k, p.k, kWidth, p.batch, p.heads, p.keys, kHalf)) return kNotEligible;
    if constexpr (kStats)
        tmap_v = tmap_k;  // statistics: no V (the map is never used)
    else if (!make_tensor_map(&tmap_v, p.v, kWidth, p.batch, p.heads, p.keys, kHalf))
        return kNotEligible;
    CUtensorMap tmap_cos = tmap_k, tmap_sin = tmap_k;
    if constexpr (kRotary) {
        const int rows = max(p.queries, p.keys);
        if (!make_table_map(&tmap_cos, p.rot_cos, p.rot_cb, p.rot_ct, rows, p.batch) ||
            !make_table_map(&tmap_sin, p.rot_sin, p.rot_sb, p.rot_st, rows, p.batch) || (p.rot_cb > 0) != (p.rot_sb > 0))
            return kNotEligible;
    }
    constexpr int bytes = shared_bytes<D, kHalf, kRotary, kTiles>();
    constexpr auto kernel = flash_forward_kernel<D, kHalf, kWidth, kRotary, kTiles, kStats, false, 1, kChained>;
    cudaError_t status = prepare_kernel<kernel>(bytes);
    if (status != cudaSuccess) return status;
    constexpr int per16 = kHalf ? 8 : 4;
    FlashArgs args{};
    args.p = p;
    args.rot_batch = p.rot_cb > 0 ? 1 : 0;
    args.cta_per_head = (p.queries + F::kCtaQueries - 1) / F::kCtaQueries;
    args.vec_out = (reinterpret_cast<uintptr_t>(p.o.data) & 15u) == 0 && p.o.sb % per16 == 0 && p.o.sh % per16 == 0 &&
                   p.o.st % per16 == 0;
    const unsigned blocks = static_cast<unsigned>(args.cta_per_head) * static_cast<unsigned>(p.heads) * static_cast<unsigned>(p.batch);
    if constexpr (kChained) {
        cudaLaunchAttribute attribute{};
        attribute.id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attribute.val.programmaticStreamSerializationAllowed = 1;
        cudaLaunchConfig_t config{};
        config.gridDim = dim3(blocks);
        config.blockDim = dim3(F::kThreads);
        config.dynamicSmemBytes = bytes;
        config.stream = stream;
        config.attrs = &attribute;
        config.numAttrs = 1;
        return cudaLaunchKernelEx(&config, kernel, args, tmap_k, tmap_v, tmap_cos, tmap_sin);
    }
    kernel<<<blocks, F::kThreads, bytes, stream>>>(args, tmap_k, tmap_v, tmap_cos, tmap_sin);
    return cudaGetLastError();
}

// d = 32 split FP32: two Q tiles per CTA share each K/V tile's conversion, but a grid of 128-query
// CTAs that fits in one wave (at most one CTA per SM) finishes sooner than half as many CTAs of
// two Q tiles. Measured on B200 (us): B2 H8 S512 23.5 -> 19.4 with one Q tile (64 CTAs);
// B8 H3 S1024 (192 one-tile CTAs, two waves) 35.8 -> 56.3, so two tiles stay there.
template <int D, bool kHalf, int kWidth = D, bool kRotary = false, bool kStats = false>
int launch(const AttentionParams &p, cudaStream_t stream) {
    int device = 0, sms = 0;
    cudaError_t status = cudaGetDevice(&device);
    if (status == cudaSuccess) status = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    if (status != cudaSuccess) return status;
    const long long one_tile_ctas = static_cast<long long>((p.queries + kQTile - 1) / kQTile) * p.heads * p.batch;
    // One-wave one-tile grids (every storage mode and width) are launched chained (kChained):
    // measured on B200, B2 H8 S512 d = 32 back to back 16.4 -> 15.6 us. Two-tile and multi-wave
    // grids are not: two-tile CTAs then start on the SMs the grid ahead left free and ran their
    // tiles ~6 % slower (B8 H3 S1024 31.1 -> 33.4 us).
    if (one_tile_ctas <= sms) return launch_tiles<D, kHalf, kWidth, kRotary, 1, kStats, true>(p, stream);
    return launch_tiles<D, kHalf, kWidth, kRotary, Forward<D, kHalf>::kQTiles, kStats>(p, stream);
}

// Prepared d = 32 forward, one or two Q tiles per CTA (the same choice as launch()): the operand
// pre-pass into `workspace`, then the forward as its programmatic dependent.
template <int kTiles, bool kRotary, int kRowThreads = 1>
int launch_prepared_tiles(const AttentionParams &p, uint8_t *workspace, cudaStream_t stream) {
    using F = Forward<32, false, kTiles, true, kRowThreads>;
    constexpr auto kernel = flash_forward_kernel<32, false, 32, kRotary, kTiles, false, true, kRowThreads>;
    constexpr int bytes = static_cast<int>(sizeof(SharedStorage<32, false, kTiles, true, kRowThreads>)) + 1024;
    static_assert(bytes <= 227 * 1024, "prepared stages fit in shared memory");
    cudaError_t status = prepare_kernel<kernel>(bytes);
    if (status != cudaSuccess) return status;
    const int tiles_per_head = (p.keys + kKeyTile - 1) / kKeyTile;
    const long long tiles = static_cast<long long>(p.batch) * p.heads * tiles_per_head;
    StageHeader *headers = reinterpret_cast<StageHeader *>(workspace + tiles * kImageBytes);
    prepare_kv_kernel<kRotary><<<static_cast<unsigned>(tiles), kPrepareThreads, 0, stream>>>(p, workspace, headers, tiles_per_head);
    status = cudaGetLastError();
    if (status != cudaSuccess) return status;
    FlashArgs args{};
    args.p = p;
    args.rot_batch = p.rot_cb > 0 ? 1 : 0;
    args.cta_per_head = (p.queries + F::kCtaQueries - 1) / F::kCtaQueries;
    args.vec_out = (reinterpret_cast<uintptr_t>(p.o.data) & 15u) == 0 && p.o.sb % 4 == 0 && p.o.sh % 4 == 0 && p.o.st % 4 == 0;
    args.images = workspace;
    args.headers = headers;
    args.tiles_per_head = tiles_per_head;
    const CUtensorMap unused{};  // the prepared kernel reads no tensor map
    cudaLaunchAttribute attribute{};
    attribute.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attribute.val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t config{};
    config.gridDim = dim3(static_cast<unsigned>(args.cta_per_head) * static_cast<unsigned>(p.heads) * static_cast<unsigned>(p.batch));
    config.blockDim = dim3(F::kThreads);
    config.dynamicSmemBytes = bytes;
    config.stream = stream;
    config.attrs = &attribute;
    config.numAttrs = 1;
    return cudaLaunchKernelEx(&config, kernel, args, unused, unused, unused, unused);
}

// The prepared d = 32 forward in the caller's workspace (prepared_forward_bytes, 128-byte aligned).
// kNotEligible when the workspace is not aligned or the problem is too large for one pre-pass grid
// (the caller then runs the forward with split warps, which needs no workspace).
template <bool kRotary>
int launch_prepared(const AttentionParams &p, void *workspace, cudaStream_t stream) {
    const long long tiles = static_cast<long long>(p.batch) * p.heads * ((p.keys + kKeyTile - 1) / kKeyTile);
    if (tiles <= 0 || tiles >= (1ll << 31) || (reinterpret_cast<uintptr_t>(workspace) & 127u) != 0) return kNotEligible;
    int device = 0, sms = 0;
    cudaError_t status = cudaGetDevice(&device);
    if (status == cudaSuccess) status = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    if (status != cudaSuccess) return status;
    const long long one_tile_ctas = static_cast<long long>((p.queries + kQTile - 1) / kQTile) * p.heads * p.batch;
    uint8_t *base = static_cast<uint8_t *>(workspace);
    // CTA form by grid size (measured on B200, us per launch, flushed): a grid of one-tile CTAs
    // that fills two CTAs per SM runs two threads per row (B4 H12 S4096 543 -> 506, C4-shaped
    // 187 -> 166); below that one thread per row, one Q tile per CTA when that grid fits in one
    // wave, else two (B8 H3 S1024: 37.1 against 39.2 with two threads per row; B1 H8 S2048
    // 45.3 against 59.6).
    if (!kRotary && one_tile_ctas >= 2ll * sms) return launch_prepared_tiles<1, false, 2>(p, base, stream);
    if (one_tile_ctas <= sms) return launch_prepared_tiles<1, kRotary>(p, base, stream);
    return launch_prepared_tiles<2, kRotary>(p, base, stream);
}

// Whether the prepared-operand forward pays for its pre-pass. The pre-pass costs a few
// microseconds whatever the shape; the forward it enables saves ~10 % per key tile. A grid that
// fits in one wave of the split-warp kernel's CTAs with fewer than 24 key tiles per window keeps
// the split-warp kernel (measured on B200, us per launch flushed / back to back, split warps vs
// prepared: B8 H3 S1024 36.3 / 30.9 vs 37.2 / 33.0; B2 H8 S512 20.5 / 16.4 vs 20.8 / 16.4;
// B1 H8 S2048 51.3 / 47.2 vs 45.3 / 39.6).
bool use_prepared(const AttentionParams &p) {
    int device = 0, sms = 0;
    if (cudaGetDevice(&device) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess)
        return false;  // no device to run on: the launch reports the error
    const long long one_tile_ctas = static_cast<long long>((p.queries + kQTile - 1) / kQTile) * p.heads * p.batch;
    const long long split_warp_ctas = one_tile_ctas <= sms ? one_tile_ctas
                                                           : static_cast<long long>((p.queries + 2 * kQTile - 1) / (2 * kQTile)) * p.heads * p.batch;
    int first = 0, last = 0;
    key_window(0, min(p.queries, 2 * kQTile), p.keys, p.radius, first, last);
    const int window_tiles = p.radius < 0 ? (p.keys + kKeyTile - 1) / kKeyTile : (last - first + kKeyTile - 1) / kKeyTile + 1;
    return split_warp_ctas > sms || window_tiles >= 24;
}

}  // namespace

long long prepared_forward_bytes(int batch, int heads, int keys) {
    const long long tiles = static_cast<long long>(batch) * heads * ((keys + kKeyTile - 1) / kKeyTile);
    return tiles * (kImageBytes + static_cast<long long>(sizeof(StageHeader)));
}

bool flash_supported(const AttentionParams &p) {
    return p.vec4 && positive_tma_strides(p.k, 4) && positive_tma_strides(p.v, 4) && (p.q.st % 4 == 0) &&
           (reinterpret_cast<uintptr_t>(p.q.data) & 15u) == 0;
}

int launch_flash_forward(const AttentionParams &p, int head_width, void *workspace, cudaStream_t stream) {
    if (head_width == 16) return launch<32, false, 16>(p, stream);
    if (head_width == 32) {
        const int status = workspace != nullptr && use_prepared(p) ? launch_prepared<false>(p, workspace, stream) : kNotEligible;
        return status != kNotEligible ? status : launch<32, false>(p, stream);
    }
    if (head_width == 64) return launch<64, false>(p, stream);
    return kNotEligible;
}

bool statistics_supported(const AttentionParams &p) {
    return p.vec4 && positive_tma_strides(p.k, 4) && (p.q.st % 4 == 0) && (reinterpret_cast<uintptr_t>(p.q.data) & 15u) == 0;
}

int launch_statistics(const AttentionParams &p, cudaStream_t stream) { return launch<32, false, 32, false, true>(p, stream); }

int launch_flash_forward_rotary(const AttentionParams &p, void *workspace, cudaStream_t stream) {
    const auto aligned = [](const float *t, long long sb, long long st) {
        return (reinterpret_cast<uintptr_t>(t) & 15u) == 0 && sb % 4 == 0 && st % 4 == 0;
    };
    if (!aligned(p.rot_cos, p.rot_cb, p.rot_ct) || !aligned(p.rot_sin, p.rot_sb, p.rot_st)) return kNotEligible;
    if ((p.rot_cb > 0) != (p.rot_sb > 0)) return kNotEligible;  // both tables per sequence, or both shared
    const int status = workspace != nullptr && use_prepared(p) ? launch_prepared<true>(p, workspace, stream) : kNotEligible;
    return status != kNotEligible ? status : launch<32, false, 32, true>(p, stream);
}

bool half_flash_supported(const AttentionParams &p) {
    const Tensor &q = p.q;
    return positive_tma_strides(p.k, 8) && positive_tma_strides(p.v, 8) && q.st % 8 == 0 && q.sh % 8 == 0 && q.sb % 8 == 0 &&
           (reinterpret_cast<uintptr_t>(q.data) & 15u) == 0;
}

int launch_half_flash_forward(const AttentionParams &p, int head_width, cudaStream_t stream) {
    if (head_width == 16) return launch<16, true>(p, stream);
    if (head_width == 32) return launch<32, true>(p, stream);
    if (head_width == 64) return launch<64, true>(p, stream);
    return kNotEligible;
}

bool tensor_maps_encodable(const AttentionParams &p, int head_width, bool half) {
    if (encode_function() == nullptr) return true;  // no driver here: nothing to ask
    CUtensorMap map_k, map_v;
    return make_tensor_map(&map_k, p.k, head_width, p.batch, p.heads, p.keys, half) &&
           make_tensor_map(&map_v, p.v, head_width, p.batch, p.heads, p.keys, half);
}

const char *half_kernel_name(int head_width) {
    return head_width == 16 ? "tcgen05-f16-flash-d16" : head_width == 32 ? "tcgen05-f16-flash-d32" : "tcgen05-f16-flash-d64";
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

const char *kernel_name(const AttentionParams &p, int head_width, bool workspace) {
    if (head_width == 64) return "tcgen05-f16x2-flash-d64";
    if (head_width == 16) return "tcgen05-f16x2-flash-d16";
    return workspace && use_prepared(p) ? "tcgen05-f16x2-flash-d32-prepared" : "tcgen05-f16x2-flash-d32";
}

#ifdef RK_WAIT_TEST
// Wait-test build only: makes CTA 0 of the next flash forwards withhold key tile `tile` (-1 to
// stop). Returns the cudaMemcpyToSymbol status.
extern "C" __attribute__((visibility("default"))) int rocmkernels_attention_test_withhold_tile(int tile) {
    return cudaMemcpyToSymbol(g_withheld_tile, &tile, sizeof(tile));
}
#endif

#ifdef RK_TC_TRACE
extern "C" __attribute__((visibility("default"))) int rocmkernels_attention_trace(long long *out, int capacity) {
    const int count = kTraceTiles * kTraceEvents;
    if (capacity < count) return -1;
    if (cudaMemcpyFromSymbol(out, g_trace, sizeof(long long) * count) != cudaSuccess) return -2;
    if (capacity >= count + 64 && cudaMemcpyFromSymbol(out + count, g_warp_trace, sizeof(long long) * 64) != cudaSuccess) return -3;
    return count;
}

// Per-CTA globaltimer stamps (kTraceCtas x 5: entry, set-up done, results written, exit, SM).
extern "C" __attribute__((visibility("default"))) int rocmkernels_attention_cta_trace(unsigned long long *out, int capacity) {
    const int count = kTraceCtas * 5;
    if (capacity < count) return -1;
    if (cudaMemcpyFromSymbol(out, g_cta_trace, sizeof(unsigned long long) * count) != cudaSuccess) return -2;
    return count;
}
#endif

const char *build_info() {
    return "sm_100a; tcgen05-f16x2-flash-d16/d32/d64 forward (TMA + TMEM, split FP16 operands, double-buffered S, tensor-core row "
           "sums; one or two Q tiles per CTA by grid size; a statistics-only mode for d32); tcgen05-f16-flash-d16/d32/d64 generic "
           "forward for FP16 storage; tcgen05 split-FP16 backward d32/d64 "
           "(query-major delta+dQ, key-major dK/dV); simt-fp32 d16/d32/d64 forward (FP32 or FP16 storage), d32/d64 backward";
}

}  // namespace tc
}  // namespace rk
