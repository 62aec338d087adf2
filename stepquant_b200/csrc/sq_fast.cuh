// Device helpers shared by the register-resident decode kernels (sq_fast.cu,
// sq_fast_kda.cu): cp.async staging, packed f32x2 arithmetic whose roundings
// match the scalar IEEE operations, division by fp16 scales, rounding on the
// FMA pipe.  Included by each kernel file (internal linkage).
#pragma once

#include "sq_tile.cuh"

namespace sq {
namespace {

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async4(void *smem, const void *gmem) {
    const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async8(void *smem, const void *gmem) {
    const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

// Packed f32x2 arithmetic (sm_100): two independent IEEE round-to-nearest lanes.
// Caution: ptxas (CUDA 12.9) fuses a packed multiply whose result feeds a
// packed add into one packed FMA even with -fmad=false and explicit .rn, which
// changes the rounding.  Every sum the quantizer must reproduce bit for bit is
// therefore accumulated with scalar __fadd_rn (ptxas keeps those separate).
__device__ __forceinline__ float2 pmul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 pfma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 add_lanes(float2 a, float2 b) { return make_float2(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y)); }

// Correctly rounded a / b for b an fp16 value (see the header comment), rb = RN(1/b).
__device__ __forceinline__ float div_fp16(float a, float b, float rb) {
    const float q = __fmul_rn(a, rb);
    const float r = __fmaf_rn(-q, b, a);
    return __fmaf_rn(r, rb, q);
}

template <bool SLOW>
__device__ __forceinline__ float divide(float a, float b, float rb) {
    return SLOW ? __fdiv_rn(a, b) : div_fp16(a, b, rb);
}

// Two lanes of div_fp16 in packed f32x2 arithmetic (each lane rounds as the
// scalar operation does); nb = -b.
template <bool SLOW>
__device__ __forceinline__ float2 divide2(float2 a, float2 b, float2 rb, float2 nb) {
    if (SLOW) return make_float2(__fdiv_rn(a.x, b.x), __fdiv_rn(a.y, b.y));
    const float2 q = pmul2(a, rb);
    const float2 r = pfma2(q, nb, a);
    return pfma2(r, rb, q);
}

// Round-half-even to an integer on the FMA pipe: for |y| <= 2^22,
// (y + 1.5*2^23) rounds y at the unit place (ties to even: 1.5*2^23 is even),
// and subtracting the constant back is exact.  The integer also sits in the
// low mantissa bits of the sum (two's complement low byte for |y| < 128).
constexpr float kRound = 12582912.f;  // 1.5 * 2^23
__device__ __forceinline__ float2 round_sum2(float2 y) { return add_lanes(y, make_float2(kRound, kRound)); }
__device__ __forceinline__ float2 clamp2(float2 y, float q) {
    return make_float2(fminf(fmaxf(y.x, -q), q), fminf(fmaxf(y.y, -q), q));
}

__device__ __forceinline__ float2 lo2(float4 v) { return make_float2(v.x, v.y); }
__device__ __forceinline__ float2 hi2(float4 v) { return make_float2(v.z, v.w); }


// ---- tensor memory as state storage --------------------------------------
// A thread keeps its state values in its own tensor-memory lane (32x32b
// accesses: warp w reaches lanes 32 (w % 4) .. +31, thread i of the warp lane
// 32 (w % 4) + i), so no two threads exchange data through it and no fences
// beyond the allocation's are needed.  Loads tie their destination registers
// to the wait, so no use can be scheduled ahead of it.
__device__ __forceinline__ void tm_alloc(uint32_t *slot, uint32_t cols) {  // one full warp
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n"
                 ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(slot))), "r"(cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n");
}
__device__ __forceinline__ void tm_dealloc(uint32_t base, uint32_t cols) {  // one full warp
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(base), "r"(cols));
}
__device__ __forceinline__ void tm_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tm_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tm_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }

// 16 consecutive fp32 columns of the thread's lane <-> v[i][h] = columns 4i + 2h, 4i + 2h + 1.
__device__ __forceinline__ void tm_ld16(uint32_t taddr, float2 (&v)[4][2]) {
    uint32_t r[16];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;\n"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
                 :: "memory");
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        v[i][0] = make_float2(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1]));
        v[i][1] = make_float2(__uint_as_float(r[4 * i + 2]), __uint_as_float(r[4 * i + 3]));
    }
}
__device__ __forceinline__ void tm_st16(uint32_t taddr, const float2 (&v)[4][2]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n"
                 ::"r"(taddr), "f"(v[0][0].x), "f"(v[0][0].y), "f"(v[0][1].x), "f"(v[0][1].y), "f"(v[1][0].x),
                   "f"(v[1][0].y), "f"(v[1][1].x), "f"(v[1][1].y), "f"(v[2][0].x), "f"(v[2][0].y), "f"(v[2][1].x),
                   "f"(v[2][1].y), "f"(v[3][0].x), "f"(v[3][0].y), "f"(v[3][1].x), "f"(v[3][1].y)
                 : "memory");
}

// Exact sum terms: a product formed by an FFMA2 with a +0 addend (the same
// rounding as the product alone; ptxas does not merge it into the following
// add) accumulated with a packed add.
__device__ __forceinline__ float2 product_term(float2 a, float2 b) { return pfma2(a, b, make_float2(0.f, 0.f)); }

}  // namespace
}  // namespace sq
