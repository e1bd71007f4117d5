// common.cuh - formats, bit conversions and small device helpers shared by the sm_100a MoE kernels.
//
// Formats (ggml, as StrataMetal stores them):
//   Q2_0  (type 42): 18 B / 64 values  = { fp16 d; u8 qs[16] }, 4 codes per byte LSB first, value (code-1)*d
//                    (include/strata/artifact/dequant.hpp:8-13, 69-78)
//   IQ2_S (type 22): 82 B / 256 values = { fp16 d; qs[32]; signs[32]; qh[8]; scales[8] }
//                    (metal/shaders/iq.metal:152-180, gguf_reader.hpp:197-199)
//   q8_1           : 36 B / 32 values  = { fp16 d; fp16 sum; int8 q[32] }  (iq.metal:597-627)
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#define SMOE_HD __host__ __device__ __forceinline__

namespace smoe {

constexpr int kQ2_0 = 42;
constexpr int kIQ2_S = 22;
constexpr int kIQ4_NL = 20;   // these four: the any-format layer path and the stage entry point (iqx.cu)
constexpr int kIQ4_XS = 23;
constexpr int kIQ3_XXS = 18;
constexpr int kIQ3_S = 21;
constexpr int kQ8Block = 36;

// Status word shared by all kernels of this library (one per device).  A kernel that gives up on a
// bounded wait records its code here; the host reads and clears it with smoe_device_status().
enum : unsigned { kDevOk = 0, kDevTimeout = 1, kDevBadId = 2 };
// The library is one translation unit (smoe_lib.cu), so the word is defined here, once.
__device__ unsigned g_smoe_status = 0;

SMOE_HD uint32_t f2u(float f) {
#ifdef __CUDA_ARCH__
    return __float_as_uint(f);
#else
    uint32_t u;
    __builtin_memcpy(&u, &f, 4);
    return u;
#endif
}

SMOE_HD float u2f(uint32_t u) {
#ifdef __CUDA_ARCH__
    return __uint_as_float(u);
#else
    float f;
    __builtin_memcpy(&f, &u, 4);
    return f;
#endif
}

// Round-to-nearest-even f32 -> bf16 bits; a NaN is passed through quieted (the rule of
// include/strata/kernels/bf16_bits.hpp:37-47).
SMOE_HD uint16_t bf16_bits(float f) {
    uint32_t i = f2u(f);
    if ((i & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t) ((i >> 16) | 64u);
    i = (i + ((i >> 16) & 1u) + 0x7FFFu) & 0xFFFF0000u;
    return (uint16_t) (i >> 16);
}

SMOE_HD float bf16_round(float f) { return u2f((uint32_t) bf16_bits(f) << 16); }

// Round-to-nearest-even f32 -> fp16 bits, subnormals kept, finite overflow -> inf, NaN stays NaN
// (IEEE binary16; the rounding rule include/strata/kernels/f16_bits.hpp:37-73 states).
SMOE_HD uint16_t f16_bits(float f) {
    const uint32_t x = f2u(f);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t rawexp = (x >> 23) & 0xFFu;
    const int e = (int) rawexp - 127 + 15;
    uint32_t man = x & 0x7FFFFFu;
    if (rawexp == 0xFFu) return (uint16_t) (sign | 0x7C00u | (man ? 0x200u : 0u));
    if (e >= 31) return (uint16_t) (sign | 0x7C00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t) sign;
        man |= 0x800000u;
        const uint32_t sh = (uint32_t) (14 - e);
        uint32_t h = (man >> sh) & 0x3FFu;
        const uint32_t rem = man & ((1u << sh) - 1u);
        const uint32_t half = 1u << (sh - 1);
        if (rem > half || (rem == half && (h & 1u))) ++h;
        return (uint16_t) (sign | h);
    }
    uint32_t h = sign | ((uint32_t) e << 10) | (man >> 13);
    const uint32_t rem = man & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
    return (uint16_t) h;
}

// Exact fp16 -> f32 (every fp16 value, subnormals included, is an f32 value).
__device__ __forceinline__ float f16_to_f32(uint16_t h) {
    float f;
    asm("{ .reg .b16 t; mov.b16 t, %1; cvt.f32.f16 %0, t; }" : "=f"(f) : "h"(h));
    return f;
}

__device__ __forceinline__ float f32_from_bf16_bits(uint16_t h) { return __uint_as_float((uint32_t) h << 16); }

// dp4a with an UNSIGNED first operand (weight codes 0..255) and a signed second (q8 activations).
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ int dp4a_ss(int a, int b, int c) {
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ------------------------------------------------------------------------------------------------
// mbarrier + 1D bulk copy (TMA without a tensor map).  Every wait is bounded.
// ------------------------------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t) __cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

// Bulk global -> shared copy; dst, src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for phase `parity` of `bar` for at most `limit_ns`; false when the limit ran out.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (global_timer_ns() - t0 > limit_ns) return false;
    }
    return true;
}

// try_wait with a suspend-time hint: a thread whose phase has not completed sleeps until it completes or the
// hint elapses, instead of spinning on the issue slots its neighbours need.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// mbar_wait_bounded built on the sleeping try_wait.
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
    if (mbar_try_wait_sleep(bar, parity, 20000u)) return true;
    const uint64_t t0 = global_timer_ns();
    while (!mbar_try_wait_sleep(bar, parity, 20000u)) {
        if (global_timer_ns() - t0 > limit_ns) return false;
    }
    return true;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Named barrier over `n` threads that also ANDs a predicate across them (every thread gets the result).
__device__ __forceinline__ bool bar_and(int id, int n, bool pred) {
    uint32_t r;
    asm volatile(
        "{ .reg .pred p, q; setp.ne.u32 p, %1, 0; bar.red.and.pred q, %2, %3, p; selp.u32 %0, 1, 0, q; }"
        : "=r"(r)
        : "r"((uint32_t) pred), "r"(id), "r"(n)
        : "memory");
    return r != 0;
}

constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s: far above any legal copy, far below a hang

// ------------------------------------------------------------------------------------------------
// tcgen05 (5th-generation tensor cores): shared-memory matrix descriptors, kind::f16 MMA, tensor memory.
// ------------------------------------------------------------------------------------------------

// Shared-memory matrix descriptor, no swizzle: start >> 4 at [0,14), leading byte offset >> 4 at [16,30),
// stride byte offset >> 4 at [32,46), descriptor version 1 at bit 46, base offset 0, layout type 0.
// K-major canonical layout ((8,m),(8 elements,2)) : ((16 B, SBO), (1, LBO)): core matrices of 8 rows x 16 B,
// LBO between core matrices adjacent in K, SBO between 8-row groups.
__device__ __forceinline__ uint64_t umma_desc(const void* smem_ptr, uint32_t lbo, uint32_t sbo) {
    const uint32_t a = smem_addr(smem_ptr);
    return (uint64_t) ((a >> 4) & 0x3FFFu) | ((uint64_t) ((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t) ((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

// Instruction descriptor of kind::f16 with f16 A and B, f32 accumulator, both K-major, M x N.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int M, int N) {
    return (1u << 4) | ((uint32_t) (N >> 3) << 17) | ((uint32_t) (M >> 4) << 24);
}

// D[tmem] (+)= A[smem] * B[smem]^T, issued by one thread.
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(
            d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T: A in tensor memory (lane = row, two fp16 per 32-bit column, K-major).
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p; }" ::"r"(
            d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// The mbarrier completes one arrival once every MMA this thread issued before has finished.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {  // whole warp
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst)),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {  // whole warp
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {  // whole warp
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 8 consecutive 32-bit columns of this thread's tensor-memory lane (the warp reads lanes 32 (warp % 4) + 0..31).
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr)
                 : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// tcgen05.ld completes asynchronously: its destination registers hold the data only after tcgen05.wait::ld.  The
// compiler sees the load's outputs as ready at once, so the wait names the loaded registers (in and out): no use
// of them can be scheduled before it.
#define SMOE_R8(a, o) "+r"(a[o + 0]), "+r"(a[o + 1]), "+r"(a[o + 2]), "+r"(a[o + 3]), "+r"(a[o + 4]), "+r"(a[o + 5]), \
                      "+r"(a[o + 6]), "+r"(a[o + 7])
__device__ __forceinline__ void tmem_wait_ld8x4(uint32_t (&a)[8], uint32_t (&b)[8], uint32_t (&c)[8], uint32_t (&d)[8]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;" : SMOE_R8(a, 0), SMOE_R8(b, 0), SMOE_R8(c, 0), SMOE_R8(d, 0)::"memory");
}
__device__ __forceinline__ void tmem_wait_ld32(uint32_t (&a)[32]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;" : SMOE_R8(a, 0), SMOE_R8(a, 8), SMOE_R8(a, 16), SMOE_R8(a, 24)::"memory");
}

// 16 consecutive 32-bit columns of this thread's tensor-memory lane (the warp writes lanes 32 (warp % 4) + 0..31).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// tcgen05.st reads its source registers asynchronously too: the wait names them, so they stay live and unchanged
// until the store has completed.
__device__ __forceinline__ void tmem_wait_st16(uint32_t* a) {
    asm volatile("tcgen05.wait::st.sync.aligned;" : SMOE_R8(a, 0), SMOE_R8(a, 8)::"memory");
}
__device__ __forceinline__ void tmem_wait_st32(uint32_t* a) {
    asm volatile("tcgen05.wait::st.sync.aligned;" : SMOE_R8(a, 0), SMOE_R8(a, 8), SMOE_R8(a, 16), SMOE_R8(a, 24)::"memory");
}

}  // namespace smoe
