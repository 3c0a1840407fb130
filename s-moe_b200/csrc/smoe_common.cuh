// smoe_common.cuh - PTX helpers shared by the sm_100a kernels.
#pragma once
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#define SMOE_DEVINL __device__ __forceinline__

// Device-side error codes written into the context's error word.
enum : uint32_t {
    SMOE_DEVERR_NONE = 0,
    SMOE_DEVERR_MBAR_TIMEOUT = 1,   // a bulk copy never completed
    SMOE_DEVERR_SPIN_TIMEOUT = 2,   // a cross-CTA or cross-GPU wait ran out
    SMOE_DEVERR_BAD_EXPERT = 3,     // an expert id >= the layer's expert count (slot skipped)
};

// Waits without a caller-given limit (the bulk-copy completions of the
// two-kernel and grouped paths) give up after this many nanoseconds of
// %globaltimer time: far beyond any legitimate wait (microseconds), far below
// a watchdog. An iteration cap backs the clock up.
#define SMOE_WAIT_NS_DEFAULT 1000000000ull
#define SMOE_SPIN_LIMIT (1u << 26)

SMOE_DEVINL uint64_t gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

SMOE_DEVINL uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

SMOE_DEVINL uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
    // (a & b) | c
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Packed fp16 a - (1024, 1024): exact for the 1024+q / 1024+16q operands.
SMOE_DEVINL uint32_t hsub_1024(uint32_t a) {
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(0x64006400u));
    return d;
}

// Packed bf16 a - (128, 128): exact for the 128+q operands.
SMOE_DEVINL uint32_t bsub_128(uint32_t a) {
    uint32_t d;
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(0x43004300u));
    return d;
}

// D += A(16x16, bf16, row) * B(16x8, bf16, col), fp32 accumulate.
SMOE_DEVINL void mma_bf16_16816(float d[4], const uint32_t a[4], const uint32_t b[2]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// D += A(16x32, u8, row) * B(32x8, s8, col), exact int32 accumulate. No side
// effects, so not volatile: the compiler may interleave it with the loads.
SMOE_DEVINL void mma_u8s8_16832(int d[4], const uint32_t a[4], const uint32_t b[2]) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// D += A(16x16, u8, row) * B(16x8, s8, col), exact int32 accumulate.
SMOE_DEVINL void mma_u8s8_16816(int d[4], const uint32_t a[2], uint32_t b) {
    asm("mma.sync.aligned.m16n8k16.row.col.s32.u8.s8.s32 "
        "{%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(b));
}

// D += A(16x16, u8, row) * B(16x8, u8, col), s32 accumulate.
SMOE_DEVINL void mma_u8u8_16816(int d[4], const uint32_t a[2], uint32_t b) {
    asm("mma.sync.aligned.m16n8k16.row.col.s32.u8.u8.s32 "
        "{%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(b));
}

SMOE_DEVINL uint32_t pack_bf16x2(float lo, float hi) {
    const __nv_bfloat16 a = __float2bfloat16_rn(lo), b = __float2bfloat16_rn(hi);
    return uint32_t(__bfloat16_as_ushort(a)) | (uint32_t(__bfloat16_as_ushort(b)) << 16);
}

// D += A(16x16, f16, row) * B(16x8, f16, col), fp32 accumulate.
SMOE_DEVINL void mma_f16_16816(float d[4], const uint32_t a[4], const uint32_t b[2]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// D = A(16x16, f16, row) * B(16x8, f16, col), fp32, zero accumulator in.
SMOE_DEVINL void mma_f16_16816_z(float d[4], const uint32_t a[4], const uint32_t b[2]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]), "f"(0.0f));
}

// ------------------------------------------------------------- mbarrier
SMOE_DEVINL void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(bar)), "r"(count));
}
SMOE_DEVINL void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
SMOE_DEVINL void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
SMOE_DEVINL void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                 :: "r"(smem_u32(bar)), "r"(bytes) : "memory");
}
SMOE_DEVINL void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(smem_u32(bar)) : "memory");
}
SMOE_DEVINL bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}
// Bounded wait; returns false (and the caller raises the error flag) when
// the phase never completes.
// The loop is kept out of line: the many wait sites then add one try_wait
// and a call each to the hot code instead of a copy of the loop.
// Bounded by a %globaltimer deadline (absolute, ns).
static __device__ __noinline__ bool mbar_wait_until(uint64_t* bar, uint32_t parity, uint64_t deadline) {
#pragma unroll 1
    for (uint32_t i = 0; i < SMOE_SPIN_LIMIT; ++i) {
        if (mbar_try_wait(bar, parity)) return true;   // try_wait itself suspends a while
        if ((i & 15) == 15 && gtimer() > deadline) return false;
        if (i > 4096) __nanosleep(64);
    }
    return false;
}
static __device__ __noinline__ bool mbar_wait_slow(uint64_t* bar, uint32_t parity) {
    return mbar_wait_until(bar, parity, gtimer() + SMOE_WAIT_NS_DEFAULT);
}
SMOE_DEVINL bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
    return mbar_try_wait(bar, parity) || mbar_wait_slow(bar, parity);
}
// Budget of one wait: `ns` from when the wait starts, but never past `cap`
// (an absolute limit for the whole kernel). A wait that ran out thus does
// not use up the budget of the waits after it, and the kernel still ends.
struct WaitBudget {
    uint64_t ns, cap;
    SMOE_DEVINL uint64_t deadline() const {
        const uint64_t t = gtimer() + ns;
        return t < cap ? t : cap;
    }
};
SMOE_DEVINL bool mbar_wait_b(uint64_t* bar, uint32_t parity, const WaitBudget& w) {
    return mbar_try_wait(bar, parity) || mbar_wait_until(bar, parity, w.deadline());
}
// The same, setting the device error word when the wait runs out; the slow
// path is out of line, so a call site is a try_wait and a branch.
static __device__ __noinline__ void mbar_wait_flag_slow(uint64_t* bar, uint32_t parity, uint64_t ns, uint64_t cap,
                                                        uint32_t* err) {
    const WaitBudget w{ns, cap};
    if (!mbar_wait_until(bar, parity, w.deadline())) atomicCAS(err, 0u, SMOE_DEVERR_MBAR_TIMEOUT);
}
SMOE_DEVINL void mbar_wait_e(uint64_t* bar, uint32_t parity, const WaitBudget& w, uint32_t* err) {
    if (!mbar_try_wait(bar, parity)) mbar_wait_flag_slow(bar, parity, w.ns, w.cap, err);
}

// 1-D bulk copy global -> shared, completion counted on `bar` (bytes).
// dst, src 16-byte aligned; bytes a multiple of 16. No multicast.
SMOE_DEVINL void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        :: "r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

// ----------------------------------------------------------- conversions
SMOE_DEVINL float bf16_bits_to_f32(uint16_t b) { return __uint_as_float(uint32_t(b) << 16); }
SMOE_DEVINL float f16_bits_to_f32(uint16_t h) { return __half2float(__ushort_as_half(h)); }

SMOE_DEVINL uint32_t pack_half2(__half lo, __half hi) {
    return uint32_t(__half_as_ushort(lo)) | (uint32_t(__half_as_ushort(hi)) << 16);
}

SMOE_DEVINL uint32_t ld_volatile_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}
