// sm_100a primitives written as inline PTX: mbarriers with bounded waits, TMA tensor loads,
// tcgen05 TMEM allocation / loads / stores, UMMA descriptors and tcgen05.mma (kind::tf32).
//
// Encodings follow the PTX ISA for tcgen05 (shared-memory matrix descriptor: start address,
// leading/stride byte offsets in 16-byte units, version 1 at bit 46, swizzle mode at bits 61-63;
// instruction descriptor: D format at bits 4-5, A/B formats at 7-9/10-12, A/B major at 15/16,
// N/8 at bits 17-22, M/16 at bits 24-28).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace rk {
namespace tc {

// Status word for failed bounded waits (never expected; read by rocmkernels_attention_device_status).
// One copy per translation unit that includes this header.
static __device__ unsigned int g_device_status = 0;
constexpr unsigned int kStatusWaitTimeout = 1u;

// ~1 s at 2 GHz: a healthy wait is microseconds; a wait this long means a protocol bug.
constexpr long long kWaitTimeoutCycles = 1ll << 31;

__device__ __forceinline__ uint32_t smem_u32(const void *pointer) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(pointer));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(smem_u32(bar)), "r"(parity)
            : "memory");
    return done != 0;
}

// Non-blocking test of the phase with the given parity (never suspends the thread; for polling
// several barriers from one thread).
__device__ __forceinline__ bool mbar_test_wait(uint64_t *bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(smem_u32(bar)), "r"(parity)
            : "memory");
    return done != 0;
}

// Waits for the phase with the given parity to complete; gives up after kWaitTimeoutCycles,
// records kStatusWaitTimeout in g_device_status and returns false.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long start = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - start > kWaitTimeoutCycles) {
            atomicOr(&g_device_status, kStatusWaitTimeout);
            return false;
        }
    }
    return true;
}

// 4-D tiled TMA load (no multicast) completing on `bar` with complete_tx.
__device__ __forceinline__ void tma_load_4d(void *dst, const CUtensorMap *map, uint64_t *bar, int c0, int c1, int c2, int c3) {
    asm volatile(
            "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(
                    smem_u32(dst)),
            "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
            : "memory");
}

__device__ __forceinline__ void fence_proxy_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ---- TMEM -------------------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t *dst, uint32_t columns) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(columns) : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t columns) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(columns) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

#define RK_R8(i) "=r"(r[i]), "=r"(r[i + 1]), "=r"(r[i + 2]), "=r"(r[i + 3]), "=r"(r[i + 4]), "=r"(r[i + 5]), "=r"(r[i + 6]), "=r"(r[i + 7])
#define RK_W8(i) "r"(r[i]), "r"(r[i + 1]), "r"(r[i + 2]), "r"(r[i + 3]), "r"(r[i + 4]), "r"(r[i + 5]), "r"(r[i + 6]), "r"(r[i + 7])

// 32 consecutive 32-bit TMEM columns of this thread's lane (32x32b shape), load + wait in one
// statement so no use of the registers can be scheduled before the data has arrived.
__device__ __forceinline__ void tmem_load32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
            "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
            "tcgen05.wait::ld.sync.aligned;"
            : RK_R8(0), RK_R8(8), RK_R8(16), RK_R8(24)
            : "r"(taddr)
            : "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_store32(uint32_t taddr, const float (&v)[32]) {
    uint32_t r[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(v[i]);
    asm volatile(
            "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
            "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n\t"
            "tcgen05.wait::st.sync.aligned;" ::"r"(taddr),
            RK_W8(0), RK_W8(8), RK_W8(16), RK_W8(24)
            : "memory");
}

// 16 columns at a and 16 columns at b with one wait.
__device__ __forceinline__ void tmem_load16x2(uint32_t a, float (&va)[16], uint32_t b, float (&vb)[16]) {
    uint32_t r[32];
    asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%32];\n\t"
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%33];\n\t"
            "tcgen05.wait::ld.sync.aligned;"
            : RK_R8(0), RK_R8(8), RK_R8(16), RK_R8(24)
            : "r"(a), "r"(b)
            : "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        va[i] = __uint_as_float(r[i]);
        vb[i] = __uint_as_float(r[16 + i]);
    }
}

// 16 columns at a, 16 columns at b and the single column c with one wait.
__device__ __forceinline__ void tmem_load16x2_1(uint32_t a, float (&va)[16], uint32_t b, float (&vb)[16], uint32_t c,
                                                float &vc) {
    uint32_t r[33];
    asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%33];\n\t"
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%34];\n\t"
            "tcgen05.ld.sync.aligned.32x32b.x1.b32 {%32}, [%35];\n\t"
            "tcgen05.wait::ld.sync.aligned;"
            : RK_R8(0), RK_R8(8), RK_R8(16), RK_R8(24), "=r"(r[32])
            : "r"(a), "r"(b), "r"(c)
            : "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        va[i] = __uint_as_float(r[i]);
        vb[i] = __uint_as_float(r[16 + i]);
    }
    vc = __uint_as_float(r[32]);
}

// 16 columns at a and 16 columns at b, one wait for both stores.
__device__ __forceinline__ void tmem_store16x2(uint32_t a, const float *va, uint32_t b, const float *vb) {
    uint32_t r[32];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        r[i] = __float_as_uint(va[i]);
        r[16 + i] = __float_as_uint(vb[i]);
    }
    asm volatile(
            "tcgen05.st.sync.aligned.32x32b.x16.b32 [%32], {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15};\n\t"
            "tcgen05.st.sync.aligned.32x32b.x16.b32 [%33], {%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31};\n\t"
            "tcgen05.wait::st.sync.aligned;" ::RK_W8(0),
            RK_W8(8), RK_W8(16), RK_W8(24), "r"(a), "r"(b)
            : "memory");
}

// 32 columns at a and 32 columns at b, one wait for both stores.
__device__ __forceinline__ void tmem_store32x2(uint32_t a, const float *va, uint32_t b, const float *vb) {
    uint32_t r[64];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        r[i] = __float_as_uint(va[i]);
        r[32 + i] = __float_as_uint(vb[i]);
    }
    asm volatile(
            "tcgen05.st.sync.aligned.32x32b.x32.b32 [%64], {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
            "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31};\n\t"
            "tcgen05.st.sync.aligned.32x32b.x32.b32 [%65], {%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,"
            "%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63};\n\t"
            "tcgen05.wait::st.sync.aligned;" ::RK_W8(0),
            RK_W8(8), RK_W8(16), RK_W8(24), RK_W8(32), RK_W8(40), RK_W8(48), RK_W8(56), "r"(a), "r"(b)
            : "memory");
}

// 64 columns (two 32-column blocks at taddr and taddr + 32) with one wait.
__device__ __forceinline__ void tmem_load64(uint32_t taddr, float (&v)[64]) {
    uint32_t r[64];
    asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
            "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%64];\n\t"
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
            "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%65];\n\t"
            "tcgen05.wait::ld.sync.aligned;"
            : RK_R8(0), RK_R8(8), RK_R8(16), RK_R8(24), RK_R8(32), RK_R8(40), RK_R8(48), RK_R8(56)
            : "r"(taddr), "r"(taddr + 32)
            : "memory");
#pragma unroll
    for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 columns at a and 64 columns at b (two 32-column blocks) with one wait.
__device__ __forceinline__ void tmem_load32_64(uint32_t a, float (&va)[32], uint32_t b, float (&vb)[64]) {
    uint32_t r[96];
    asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
            "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%96];\n\t"
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
            "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%97];\n\t"
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%64,%65,%66,%67,%68,%69,%70,%71,%72,%73,%74,%75,%76,%77,%78,%79,"
            "%80,%81,%82,%83,%84,%85,%86,%87,%88,%89,%90,%91,%92,%93,%94,%95}, [%98];\n\t"
            "tcgen05.wait::ld.sync.aligned;"
            : RK_R8(0), RK_R8(8), RK_R8(16), RK_R8(24), RK_R8(32), RK_R8(40), RK_R8(48), RK_R8(56), RK_R8(64),
              RK_R8(72), RK_R8(80), RK_R8(88)
            : "r"(a), "r"(b), "r"(b + 32)
            : "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) va[i] = __uint_as_float(r[i]);
#pragma unroll
    for (int i = 0; i < 64; ++i) vb[i] = __uint_as_float(r[32 + i]);
}

#undef RK_R8
#undef RK_W8

// ---- UMMA descriptors and MMA -----------------------------------------------------------------
// Shared-memory descriptor of a 128-byte-swizzled operand whose 8-row x 128-byte atoms are
// stacked every 1024 bytes (the layout a 128B-swizzled TMA box of 32 FP32 columns produces).
__device__ __forceinline__ uint64_t sw128_descriptor(uint32_t smem_byte_address) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_byte_address & 0x3FFFFu) >> 4);  // start address
    d |= static_cast<uint64_t>(1) << 16;                               // leading byte offset (unused by SW128)
    d |= static_cast<uint64_t>(1024 >> 4) << 32;                       // stride byte offset: 8 rows x 128 B
    d |= static_cast<uint64_t>(1) << 46;                               // descriptor version (sm_100)
    d |= static_cast<uint64_t>(2) << 61;                               // SWIZZLE_128B
    return d;
}

// Instruction descriptor: F16 x F16 -> F32 (kind::f16), M x N, A and B K-major.
__host__ __device__ constexpr uint32_t f16_instr_desc(int m, int n) {
    return (1u << 4) | (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

// D(tmem) (+)= A(tmem, fp16 pairs per 32-bit column) x B(smem descriptor, fp16), one thread.
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
            "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
            : "memory");
}

// Instruction descriptor: TF32 x TF32 -> F32, M x N, A K-major, B K-major or MN-major.
__host__ __device__ constexpr uint32_t tf32_instr_desc(int m, int n, bool b_mn_major) {
    return (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(b_mn_major) << 16) |
           (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

// D(tmem) (+)= A(tmem) x B(smem descriptor), issued by one thread.
__device__ __forceinline__ void mma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
            "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
            : "memory");
}

// Arrives on `bar` once every tcgen05.mma issued so far by this thread has completed.
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Warp-collective forms: the whole warp executes the call with warp-uniform operands and one
// lane chosen by elect.sync issues the instruction. Issuing from a full warp keeps the operand
// arithmetic on the uniform datapath; a single lane computing them itself needs several issue
// slots per MMA, which busy warps on the same sub-partition take (measured: 33 cycles per
// M128 N64 K16 MMA this way, 160 from a lone lane beside two FFMA-bound warps).
__device__ __forceinline__ void mma_f16_ts_warp(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                uint32_t accumulate) {
    asm volatile(
            "{\n\t.reg .pred e, p;\n\t"
            "elect.sync _|e, 0xffffffff;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
            "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
            : "memory");
}

__device__ __forceinline__ void mma_commit_warp(uint64_t *bar) {
    asm volatile(
            "{\n\t.reg .pred e;\n\t"
            "elect.sync _|e, 0xffffffff;\n\t"
            "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(smem_u32(bar))
            : "memory");
}

// Bounded wait by every lane of a warp; true only if every lane saw the phase complete.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t *bar, uint32_t parity) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity));
}

// Non-blocking test by every lane; true only if every lane saw the phase complete.
__device__ __forceinline__ bool mbar_test_wait_warp(uint64_t *bar, uint32_t parity) {
    return __all_sync(0xffffffffu, mbar_test_wait(bar, parity));
}

// Round to the nearest TF32 value (10 explicit mantissa bits, ties away from zero) with two
// integer operations: add half an ulp of the 13 dropped bits to the magnitude, clear them. The
// carry propagates into the exponent when needed; the sign bit is untouched; infinities stay
// infinite. The result is exactly representable in TF32, so the tensor core's own operand
// conversion leaves it unchanged whatever its rounding mode.
__device__ __forceinline__ float round_tf32(float x) {
    return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
}

// Packs two FP32 values as FP16 (round to nearest): a in the low half, b in the high half (the
// order a K-major fp16 operand stores consecutive elements in one 32-bit word).
__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
    uint32_t packed;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(packed) : "f"(b), "f"(a));
    return packed;
}

// max(a, b, c) in one instruction (sm_100 three-input max; NaN operands are ignored like fmaxf).
__device__ __forceinline__ float max3(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

// 2^e as FP32 for integer e, exact; 0 below the normal range, +inf above it.
__device__ __forceinline__ float exp2_int(int e) {
    return e < -126 ? 0.f : e > 127 ? __int_as_float(0x7f800000) : __int_as_float((e + 127) << 23);
}

// Exponent that brings the largest magnitude m (> 0, finite) into [2^14, 2^15): 14 - floor(log2 m),
// clamped to [-100, 100] so that 2^e and products of two such scales stay normal FP32 values. m == 0 (or not finite) gives 0.
__device__ __forceinline__ int fp16_scale_exponent(float m) {
    if (!(m > 0.f) || !isfinite(m)) return 0;
    const int exponent = ((__float_as_int(m) >> 23) & 0xff) - 127;  // floor(log2 m) for normal m
    return max(-100, min(100, 14 - exponent));
}

// x = hi + lo with hi = round_tf32(x) and lo = x - hi exact in FP32 (|lo| <= 2^-11 |x|). The
// tensor core keeps the top 11 significant bits of lo, so hi*b + lo*b carries about 22 bits.
__device__ __forceinline__ void split_tf32(float x, float &hi, float &lo) {
    hi = round_tf32(x);
    lo = x - hi;
}

}  // namespace tc
}  // namespace rk
