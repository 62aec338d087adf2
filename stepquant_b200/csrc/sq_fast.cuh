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


// Exact sum terms: a product formed by an FFMA2 with a +0 addend (the same
// rounding as the product alone; ptxas does not merge it into the following
// add) accumulated with a packed add.
__device__ __forceinline__ float2 product_term(float2 a, float2 b) { return pfma2(a, b, make_float2(0.f, 0.f)); }

}  // namespace
}  // namespace sq
