// Device helpers shared by the stepquant_b200 kernels.
//
// Exactness rules (the quantizer must reproduce the reference fit_state bits):
//  * the library is compiled with -fmad=false, so a*b+c is never contracted;
//    fused multiply-adds are written explicitly (fmaf) only where the result
//    feeds a toleranced value (the recurrent update), never in the quantizer;
//  * divisions, square roots and reciprocals are the IEEE round-to-nearest
//    forms (__fdiv_rn, __fsqrt_rn, __frcp_rn);
//  * the two fp32 sums of fit_state follow torch 2.11's CPU summation order
//    (aten SumKernel cascade_sum with 8-lane vectors), restated below.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/stepquant_b200.h"

namespace sq {

constexpr int kThreads = 256;
constexpr int kMaxDim = 128;
constexpr int kMaxGroups = 32;

// ---------------------------------------------------------------------------
// dtype access
// ---------------------------------------------------------------------------
__device__ __forceinline__ float load_as_float(const void *p, int dtype, int64_t i) {
    if (dtype == SQ_F32) return static_cast<const float *>(p)[i];
    if (dtype == SQ_BF16) return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i]);
    return __half2float(static_cast<const __half *>(p)[i]);
}

__device__ __forceinline__ void store_from_float(void *p, int dtype, int64_t i, float x) {
    if (dtype == SQ_F32) {
        static_cast<float *>(p)[i] = x;
    } else if (dtype == SQ_BF16) {
        static_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(x);
    } else {
        static_cast<__half *>(p)[i] = __float2half_rn(x);
    }
}

// ---------------------------------------------------------------------------
// fp16 scales (quantization.py:49-51): clamp to [2^-24, 65504], round to fp16.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float fp16_scale(float x) {
    x = fminf(fmaxf(x, 5.9604644775390625e-8f), 65504.0f);
    return __half2float(__float2half_rn(x));
}

__device__ __forceinline__ uint16_t half_bits(float x) {
    return __half_as_ushort(__float2half_rn(x));
}

__device__ __forceinline__ float half_at(const uint8_t *base, int64_t byte_offset) {
    return __half2float(*reinterpret_cast<const __half *>(base + byte_offset));
}

__device__ __forceinline__ void put_half(uint8_t *base, int64_t byte_offset, float x) {
    *reinterpret_cast<__half *>(base + byte_offset) = __float2half_rn(x);
}

// ---------------------------------------------------------------------------
// torch CPU summation order
//
// cascade(size, item): aten multi_row_sum for one accumulator lane.  Blocks of
// 2^level_power (>= 16) consecutive items accumulate in order; each finished
// block is carried into level 1 (and higher levels when their bit pattern
// says so); the levels are added back at the end.
// row_sum(size, item): aten row_sum: four interleaved cascades over
// item(4i+k), tail items into the first, then the four partials in order.
// ---------------------------------------------------------------------------
__device__ __forceinline__ int ceil_log2(int x) {
    int r = 0;
    while ((1 << r) < x) ++r;
    return r;
}

template <class Item>
__device__ __forceinline__ float torch_cascade(int size, Item item) {
    const int level_power = max(4, ceil_log2(size) / 4);
    const int level_step = 1 << level_power;
    const int level_mask = level_step - 1;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    int i = 0;
    while (i + level_step <= size) {
        for (int j = 0; j < level_step; ++j, ++i) acc[0] = __fadd_rn(acc[0], item(i));
        for (int j = 1; j < 4; ++j) {
            acc[j] = __fadd_rn(acc[j], acc[j - 1]);
            acc[j - 1] = 0.f;
            if (i & (level_mask << (j * level_power))) break;
        }
    }
    for (; i < size; ++i) acc[0] = __fadd_rn(acc[0], item(i));
    for (int j = 1; j < 4; ++j) acc[0] = __fadd_rn(acc[0], acc[j]);
    return acc[0];
}

template <class Item>
__device__ __forceinline__ float torch_row_sum(int size, Item item) {
    const int size_ilp = size / 4;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    if (size_ilp > 0) {
#pragma unroll
        for (int k = 0; k < 4; ++k) acc[k] = torch_cascade(size_ilp, [&](int i) { return item(4 * i + k); });
    }
    for (int i = size_ilp * 4; i < size; ++i) acc[0] = __fadd_rn(acc[0], item(i));
    float total = acc[0];
    for (int k = 1; k < 4; ++k) total = __fadd_rn(total, acc[k]);
    return total;
}

// Sum of item(0..n-1) as torch sums a contiguous row of n fp32 values
// (x.abs().mean(-1) in fit_state).  n >= 8: eight vector lanes, lane l sums
// item(8m + l) with row_sum over m, then the lanes are added in order.
template <class Item>
__device__ __forceinline__ float torch_inner_sum(int n, Item item) {
    if (n >= 8) {
        const int nv = n / 8;
        float total = 0.f;
        for (int lane = 0; lane < 8; ++lane)
            total = __fadd_rn(total, torch_row_sum(nv, [&](int m) { return item(8 * m + lane); }));
        return total;
    }
    return torch_row_sum(n, item);
}

// Sum over the key axis of a contiguous [K, V] plane for one column, as torch
// sums (.sum(-2)) with V columns: cascade over K for V >= 32 or V < 8,
// row_sum over K for 8 <= V < 32.
template <class Item>
__device__ __forceinline__ float torch_outer_sum(int keys, int values, Item item) {
    if (values >= 8 && values < 32) return torch_row_sum(keys, item);
    return torch_cascade(keys, item);
}

// ---------------------------------------------------------------------------
// page codes
// ---------------------------------------------------------------------------
// Little-endian code of `bits` width starting at bit `bitpos` of `p`.
__device__ __forceinline__ uint32_t read_code(const uint8_t *p, uint32_t bitpos, int bits) {
    const uint8_t *q = p + (bitpos >> 3);
    const uint32_t shift = bitpos & 7u;
    uint32_t v = q[0];
    if (shift + bits > 8u) v |= uint32_t(q[1]) << 8;
    return (v >> shift) & ((1u << bits) - 1u);
}

// Byte offset of value v of the fp16 pivot row at `off`: packed pages keep the
// row's values in tiles `stride` apart (pool.py:44-52); byte-carrier pages
// store the row contiguously (pool.py:33-41).
__device__ __forceinline__ int64_t pivot_at(int off, int v, int tile, int stride, bool bytes) {
    return bytes ? int64_t(off) + 2 * v : int64_t(off) + int64_t(v / tile) * stride + 2 * (v % tile);
}

__device__ __forceinline__ float qmax_of(int bits, bool gdn) {
    if (gdn && bits == 2) return 3.f;
    const int b = bits > 8 ? 8 : bits;
    return float((1 << (b - 1)) - 1);
}

__device__ __forceinline__ float norm_of(int bits, bool kda) {
    const int b = bits > 8 ? 8 : bits;
    return kda ? float(1 << (8 - b)) : 1.f;
}

// Signed level of a stored code (fused.py:32-40): offset binary, GDN 2-bit
// levels {-3,-1,1,3}; KDA scales the level by 2^(8-b).
__device__ __forceinline__ float level_of(uint32_t code, int bits, bool kda) {
    if (!kda && bits == 2) return 2.f * float(code) - 3.f;
    float z = float(int(code) - ((1 << (bits - 1)) - 1));
    return kda ? z * float(1 << (8 - bits)) : z;
}

__device__ __forceinline__ uint32_t code_of(float z, int bits, bool kda) {
    const int zi = int(z);
    if (!kda && bits == 2) return uint32_t((zi + 3) / 2);
    return uint32_t(zi + ((1 << (bits - 1)) - 1));
}

__device__ __forceinline__ void flag(int32_t *status, int bit) {
    if (status) atomicOr(status, bit);
}

// Block-wide sum of one float per thread over kThreads threads.
__device__ __forceinline__ float block_sum(float v, float *scratch32) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) scratch32[warp] = v;
    __syncthreads();
    float t = 0.f;
    if (threadIdx.x < 32) {
        t = lane < (kThreads / 32) ? scratch32[lane] : 0.f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        if (lane == 0) scratch32[0] = t;
    }
    __syncthreads();
    t = scratch32[0];
    __syncthreads();
    return t;
}

}  // namespace sq
