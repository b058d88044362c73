// sm_100a primitives written as inline PTX: mbarriers with bounded waits, TMA tensor loads,
// tcgen05 TMEM allocation / loads / stores, UMMA descriptors and warp-issued tcgen05.mma (kind::f16).
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
// The wait-test build of the library (RK_WAIT_TEST, librocmkernels_attention_waittest.so, used
// only by tests/test_wait_timeout_gpu.py) gives up after ~0.5 ms instead, so that a test can make
// a wait run out quickly.
#ifdef RK_WAIT_TEST
constexpr long long kWaitTimeoutCycles = 1ll << 20;
#else
constexpr long long kWaitTimeoutCycles = 1ll << 31;
#endif

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

// try_wait with a suspend-time hint: a thread whose phase is not complete is suspended until it
// completes or `hint_ns` elapse, instead of returning after the default, short interval.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t *bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t done;
    asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
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

// mbar_wait for a warp that waits long and shares its sub-partition with busy warps: the polls
// suspend (up to 20 us each, woken by the phase's completion) instead of spinning, so they take
// no issue slots from the other warps. Same bound and status word as mbar_wait.
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t *bar, uint32_t parity) {
    const long long start = clock64();
    while (!mbar_try_wait_sleep(bar, parity, 20000u)) {
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

// 2-D tiled TMA load (no multicast) completing on `bar` with complete_tx.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar, int c0, int c1) {
    asm volatile(
            "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
                    smem_u32(dst)),
            "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
            : "memory");
}

// Contiguous bulk copy global -> shared (no multicast) completing on `bar` with complete_tx;
// both addresses 16-byte aligned, `bytes` a multiple of 16.
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
                 "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
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

// 16 columns at each of six addresses with one wait.
__device__ __forceinline__ void tmem_load16x6(const uint32_t (&at)[6], float (&v)[6][16]) {
    uint32_t r[96];
    asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%96];\n\t"
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%97];\n\t"
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47}, [%98];\n\t"
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%99];\n\t"
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%64,%65,%66,%67,%68,%69,%70,%71,%72,%73,%74,%75,%76,%77,%78,%79}, [%100];\n\t"
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%80,%81,%82,%83,%84,%85,%86,%87,%88,%89,%90,%91,%92,%93,%94,%95}, [%101];\n\t"
            "tcgen05.wait::ld.sync.aligned;"
            : RK_R8(0), RK_R8(8), RK_R8(16), RK_R8(24), RK_R8(32), RK_R8(40), RK_R8(48), RK_R8(56), RK_R8(64), RK_R8(72),
              RK_R8(80), RK_R8(88)
            : "r"(at[0]), "r"(at[1]), "r"(at[2]), "r"(at[3]), "r"(at[4]), "r"(at[5])
            : "memory");
#pragma unroll
    for (int k = 0; k < 6; ++k)
#pragma unroll
        for (int i = 0; i < 16; ++i) v[k][i] = __uint_as_float(r[16 * k + i]);
}

// 8 columns at a and 8 columns at b with one wait.
__device__ __forceinline__ void tmem_load8x2(uint32_t a, float (&va)[8], uint32_t b, float (&vb)[8]) {
    uint32_t r[16];
    asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%16];\n\t"
            "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%8,%9,%10,%11,%12,%13,%14,%15}, [%17];\n\t"
            "tcgen05.wait::ld.sync.aligned;"
            : RK_R8(0), RK_R8(8)
            : "r"(a), "r"(b)
            : "memory");
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        va[i] = __uint_as_float(r[i]);
        vb[i] = __uint_as_float(r[8 + i]);
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

// 32 columns at a and the single column b with one wait.
__device__ __forceinline__ void tmem_load32_1(uint32_t a, float (&va)[32], uint32_t b, float &vb) {
    uint32_t r[33];
    asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
            "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%33];\n\t"
            "tcgen05.ld.sync.aligned.32x32b.x1.b32 {%32}, [%34];\n\t"
            "tcgen05.wait::ld.sync.aligned;"
            : RK_R8(0), RK_R8(8), RK_R8(16), RK_R8(24), "=r"(r[32])
            : "r"(a), "r"(b)
            : "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) va[i] = __uint_as_float(r[i]);
    vb = __uint_as_float(r[32]);
}

// 16 columns at a and the single column b with one wait.
__device__ __forceinline__ void tmem_load16_1(uint32_t a, float (&va)[16], uint32_t b, float &vb) {
    uint32_t r[17];
    asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%17];\n\t"
            "tcgen05.ld.sync.aligned.32x32b.x1.b32 {%16}, [%18];\n\t"
            "tcgen05.wait::ld.sync.aligned;"
            : RK_R8(0), RK_R8(8), "=r"(r[16])
            : "r"(a), "r"(b)
            : "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) va[i] = __uint_as_float(r[i]);
    vb = __uint_as_float(r[16]);
}

// 32 columns at a with one wait.
__device__ __forceinline__ void tmem_load32(uint32_t a, float (&va)[32]) {
    uint32_t r[32];
    asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
            "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
            "tcgen05.wait::ld.sync.aligned;"
            : RK_R8(0), RK_R8(8), RK_R8(16), RK_R8(24)
            : "r"(a)
            : "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) va[i] = __uint_as_float(r[i]);
}

// 16 columns at a with one wait.
__device__ __forceinline__ void tmem_load16(uint32_t a, float (&va)[16]) {
    uint32_t r[16];
    asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n\t"
            "tcgen05.wait::ld.sync.aligned;"
            : RK_R8(0), RK_R8(8)
            : "r"(a)
            : "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) va[i] = __uint_as_float(r[i]);
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

// 8 columns at a and 8 columns at b without waiting: the registers are consumed at issue; the
// data reaches TMEM by the next tmem_wait_store().
__device__ __forceinline__ void tmem_store8x2_async(uint32_t a, const float *va, uint32_t b, const float *vb) {
    asm volatile(
            "tcgen05.st.sync.aligned.32x32b.x8.b32 [%16], {%0,%1,%2,%3,%4,%5,%6,%7};\n\t"
            "tcgen05.st.sync.aligned.32x32b.x8.b32 [%17], {%8,%9,%10,%11,%12,%13,%14,%15};" ::"r"(__float_as_uint(va[0])),
            "r"(__float_as_uint(va[1])), "r"(__float_as_uint(va[2])), "r"(__float_as_uint(va[3])), "r"(__float_as_uint(va[4])),
            "r"(__float_as_uint(va[5])), "r"(__float_as_uint(va[6])), "r"(__float_as_uint(va[7])), "r"(__float_as_uint(vb[0])),
            "r"(__float_as_uint(vb[1])), "r"(__float_as_uint(vb[2])), "r"(__float_as_uint(vb[3])), "r"(__float_as_uint(vb[4])),
            "r"(__float_as_uint(vb[5])), "r"(__float_as_uint(vb[6])), "r"(__float_as_uint(vb[7])), "r"(a), "r"(b)
            : "memory");
}

// 8 columns at a without waiting (see tmem_store8x2_async).
__device__ __forceinline__ void tmem_store8_async(uint32_t a, const float *va) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%8], {%0,%1,%2,%3,%4,%5,%6,%7};" ::"r"(__float_as_uint(va[0])),
                 "r"(__float_as_uint(va[1])), "r"(__float_as_uint(va[2])), "r"(__float_as_uint(va[3])),
                 "r"(__float_as_uint(va[4])), "r"(__float_as_uint(va[5])), "r"(__float_as_uint(va[6])),
                 "r"(__float_as_uint(va[7])), "r"(a)
                 : "memory");
}

__device__ __forceinline__ void tmem_wait_store() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

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

// The same with B MN-major (bit 16): B's N elements are contiguous for each K index.
__host__ __device__ constexpr uint32_t f16_instr_desc_b_mn(int m, int n) { return f16_instr_desc(m, n) | (1u << 16); }

// Shared-memory descriptor of an MN-major 128B-swizzled operand: for each K index a 128-byte row
// of 64 consecutive MN elements, eight K rows per 1024-byte swizzle atom, the atoms of
// consecutive K groups every 1024 bytes (stride byte offset) and further 64-element MN chunks
// every `mn_chunk_bytes` (leading byte offset) -- the canonical layout
// Swizzle<3,4,3> o ((8,n),(8,k)):((1,LBO),(8,SBO)) in 16-byte units. A K=16 step of FP16 is two
// K groups: 2048 bytes.
__device__ __forceinline__ uint64_t sw128_mn_descriptor(uint32_t smem_byte_address, uint32_t mn_chunk_bytes) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_byte_address & 0x3FFFFu) >> 4);  // start address
    d |= static_cast<uint64_t>(mn_chunk_bytes >> 4) << 16;             // leading byte offset: next MN chunk
    d |= static_cast<uint64_t>(1024 >> 4) << 32;                       // stride byte offset: next 8 K rows
    d |= static_cast<uint64_t>(1) << 46;                               // descriptor version (sm_100)
    d |= static_cast<uint64_t>(2) << 61;                               // SWIZZLE_128B
    return d;
}

// Warp-collective forms: the whole warp executes the call with warp-uniform operands and one
// lane chosen by elect.sync issues the instructions. Issuing from a full warp keeps the operand
// arithmetic on the uniform datapath; a single lane computing them itself needs several issue
// slots per MMA, which busy warps on the same sub-partition take (measured on B200: an
// M128 N64 K16 MMA every 33 cycles this way, N/2 cycles for any N >= 48, i.e. the full rate;
// every 160 cycles from a lone lane beside two FFMA-bound warps).
__device__ __forceinline__ void mma_commit_warp(uint64_t *bar) {
    asm volatile(
            "{\n\t.reg .pred e;\n\t"
            "elect.sync _|e, 0xffffffff;\n\t"
            "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(smem_u32(bar))
            : "memory");
}

// Warp-collective: four kind::f16 MMAs into one accumulator and a commit to `bar`, issued by one
// elected lane in a single sequence (one warp instruction per MMA). The first MMA overwrites
// the accumulator when `overwrite` is set; the others accumulate.
__device__ __forceinline__ void mma4_f16_ts_commit_warp(uint32_t d, const uint32_t (&a)[4], const uint64_t (&b)[4], uint32_t idesc,
                                                        uint32_t overwrite, uint64_t *bar) {
    asm volatile(
            "{\n\t.reg .pred e, first, rest;\n\t"
            "elect.sync _|e, 0xffffffff;\n\t"
            "setp.eq.b32 first, %10, 0;\n\t"
            "setp.eq.b32 rest, %10, %10;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %5, %9, first;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%2], %6, %9, rest;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%3], %7, %9, rest;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%4], %8, %9, rest;\n\t"
            "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%11];\n\t}" ::"r"(d),
            "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "r"(idesc),
            "r"(overwrite), "r"(smem_u32(bar))
            : "memory");
}

// Warp-collective: four kind::f16 MMAs accumulating into one accumulator (no commit).
__device__ __forceinline__ void mma4_f16_ts_warp(uint32_t d, const uint32_t (&a)[4], const uint64_t (&b)[4], uint32_t idesc,
                                                 uint32_t overwrite) {
    asm volatile(
            "{\n\t.reg .pred e, first, rest;\n\t"
            "elect.sync _|e, 0xffffffff;\n\t"
            "setp.eq.b32 first, %10, 0;\n\t"
            "setp.eq.b32 rest, %10, %10;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %5, %9, first;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%2], %6, %9, rest;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%3], %7, %9, rest;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%4], %8, %9, rest;\n\t}" ::"r"(d),
            "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "r"(idesc),
            "r"(overwrite)
            : "memory");
}

// Warp-collective: one kind::f16 MMA (overwriting the accumulator when `overwrite` is set) and a
// commit to `bar`, one elected sequence.
__device__ __forceinline__ void mma1_f16_ts_commit_warp(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc, uint32_t overwrite,
                                                        uint64_t *bar) {
    asm volatile(
            "{\n\t.reg .pred e, first;\n\t"
            "elect.sync _|e, 0xffffffff;\n\t"
            "setp.eq.b32 first, %4, 0;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, first;\n\t"
            "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%5];\n\t}" ::"r"(d),
            "r"(a), "l"(b), "r"(idesc), "r"(overwrite), "r"(smem_u32(bar))
            : "memory");
}

// Warp-collective: two kind::f16 MMAs into one accumulator (the first overwriting it when
// `overwrite` is set) and a commit to `bar`, one elected sequence.
__device__ __forceinline__ void mma2_f16_ts_first_commit_warp(uint32_t d, uint32_t a0, uint32_t a1, uint64_t b0, uint64_t b1,
                                                              uint32_t idesc, uint32_t overwrite, uint64_t *bar) {
    asm volatile(
            "{\n\t.reg .pred e, first, rest;\n\t"
            "elect.sync _|e, 0xffffffff;\n\t"
            "setp.eq.b32 first, %6, 0;\n\t"
            "setp.eq.b32 rest, %6, %6;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %3, %5, first;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%2], %4, %5, rest;\n\t"
            "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%7];\n\t}" ::"r"(d),
            "r"(a0), "r"(a1), "l"(b0), "l"(b1), "r"(idesc), "r"(overwrite), "r"(smem_u32(bar))
            : "memory");
}

// Warp-collective: two accumulating kind::f16 MMAs and a commit to `bar`, one elected sequence.
__device__ __forceinline__ void mma2_f16_ts_commit_warp(uint32_t d, uint32_t a0, uint32_t a1, uint64_t b0, uint64_t b1,
                                                        uint32_t idesc, uint64_t *bar) {
    asm volatile(
            "{\n\t.reg .pred e, rest;\n\t"
            "elect.sync _|e, 0xffffffff;\n\t"
            "setp.eq.b32 rest, %5, %5;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %3, %5, rest;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%2], %4, %5, rest;\n\t"
            "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%6];\n\t}" ::"r"(d),
            "r"(a0), "r"(a1), "l"(b0), "l"(b1), "r"(idesc), "r"(smem_u32(bar))
            : "memory");
}

// Warp-collective: two accumulating kind::f16 MMAs, one elected sequence (no commit).
__device__ __forceinline__ void mma2_f16_ts_warp(uint32_t d, uint32_t a0, uint32_t a1, uint64_t b0, uint64_t b1, uint32_t idesc) {
    asm volatile(
            "{\n\t.reg .pred e, rest;\n\t"
            "elect.sync _|e, 0xffffffff;\n\t"
            "setp.eq.b32 rest, %5, %5;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %3, %5, rest;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%2], %4, %5, rest;\n\t}" ::"r"(d),
            "r"(a0), "r"(a1), "l"(b0), "l"(b1), "r"(idesc)
            : "memory");
}

// Warp-collective: four kind::f16 MMAs with A from shared memory (descriptors `a`) into one
// accumulator, the first overwriting it when `overwrite` is set (no commit).
__device__ __forceinline__ void mma4_f16_ss_warp(uint32_t d, const uint64_t (&a)[4], const uint64_t (&b)[4], uint32_t idesc,
                                                 uint32_t overwrite) {
    asm volatile(
            "{\n\t.reg .pred e, first, rest;\n\t"
            "elect.sync _|e, 0xffffffff;\n\t"
            "setp.eq.b32 first, %10, 0;\n\t"
            "setp.eq.b32 rest, %10, %10;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %5, %9, first;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %2, %6, %9, rest;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %3, %7, %9, rest;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %4, %8, %9, rest;\n\t}" ::"r"(d),
            "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "r"(idesc),
            "r"(overwrite)
            : "memory");
}

// Warp-collective: two accumulating kind::f16 MMAs with A from shared memory (no commit).
__device__ __forceinline__ void mma2_f16_ss_warp(uint32_t d, const uint64_t (&a)[2], const uint64_t (&b)[2], uint32_t idesc) {
    asm volatile(
            "{\n\t.reg .pred e, rest;\n\t"
            "elect.sync _|e, 0xffffffff;\n\t"
            "setp.eq.b32 rest, %5, %5;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %3, %5, rest;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %2, %4, %5, rest;\n\t}" ::"r"(d),
            "l"(a[0]), "l"(a[1]), "l"(b[0]), "l"(b[1]), "r"(idesc)
            : "memory");
}

// Warp-collective: two accumulating kind::f16 MMAs with A from shared memory and a commit to
// `bar`, one elected sequence.
__device__ __forceinline__ void mma2_f16_ss_commit_warp(uint32_t d, const uint64_t (&a)[2], const uint64_t (&b)[2], uint32_t idesc,
                                                        uint64_t *bar) {
    asm volatile(
            "{\n\t.reg .pred e, rest;\n\t"
            "elect.sync _|e, 0xffffffff;\n\t"
            "setp.eq.b32 rest, %5, %5;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %3, %5, rest;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %2, %4, %5, rest;\n\t"
            "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%6];\n\t}" ::"r"(d),
            "l"(a[0]), "l"(a[1]), "l"(b[0]), "l"(b[1]), "r"(idesc), "r"(smem_u32(bar))
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

// mbar_wait_sleep by every lane of a warp; true only if every lane saw the phase complete.
__device__ __forceinline__ bool mbar_wait_sleep_warp(uint64_t *bar, uint32_t parity) {
    return __all_sync(0xffffffffu, mbar_wait_sleep(bar, parity));
}

// Programmatic dependent launch. A grid launched with programmatic stream serialization may start
// while the grid before it in the stream still runs; grid_dependency_wait() returns once that grid
// has completed and its memory operations are visible (immediately for a grid launched without
// the attribute). launch_dependents() lets the next such grid be scheduled once every CTA of this
// grid has executed it or exited; it orders no memory (the dependent still waits for completion).
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// Packs two FP32 values as FP16 (round to nearest): a in the low half, b in the high half (the
// order a K-major fp16 operand stores consecutive elements in one 32-bit word).
__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
    uint32_t packed;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(packed) : "f"(b), "f"(a));
    return packed;
}

// The two FP16 halves of a packed pair as FP32 (low half in .x), exact.
__device__ __forceinline__ float2 unpack_half2(uint32_t packed) {
    float2 r;
    asm("{\n\t.reg .f16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\tcvt.f32.f16 %0, lo;\n\tcvt.f32.f16 %1, hi;\n\t}"
        : "=f"(r.x), "=f"(r.y)
        : "r"(packed));
    return r;
}

// Packed FP32 pairs (sm_100 f32x2 instructions: one issue for two lanes of work, IEEE results
// identical to the scalar forms).
__device__ __forceinline__ float2 fma_f32x2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n\t.reg .b64 x, y, z, w;\n\t"
        "mov.b64 x, {%2, %3};\n\tmov.b64 y, {%4, %5};\n\tmov.b64 z, {%6, %7};\n\t"
        "fma.rn.f32x2 w, x, y, z;\n\tmov.b64 {%0, %1}, w;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}
__device__ __forceinline__ float2 add_f32x2(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 x, y, w;\n\t"
        "mov.b64 x, {%2, %3};\n\tmov.b64 y, {%4, %5};\n\t"
        "add.rn.f32x2 w, x, y;\n\tmov.b64 {%0, %1}, w;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}
__device__ __forceinline__ float2 mul_f32x2(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 x, y, w;\n\t"
        "mov.b64 x, {%2, %3};\n\tmov.b64 y, {%4, %5};\n\t"
        "mul.rn.f32x2 w, x, y;\n\tmov.b64 {%0, %1}, w;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}
__device__ __forceinline__ float2 sub_f32x2(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 x, y, w;\n\t"
        "mov.b64 x, {%2, %3};\n\tmov.b64 y, {%4, %5};\n\t"
        "sub.rn.f32x2 w, x, y;\n\tmov.b64 {%0, %1}, w;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
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

}  // namespace tc
}  // namespace rk
