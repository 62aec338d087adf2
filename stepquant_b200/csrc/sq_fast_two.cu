// Register / tensor-memory kernels for GDN 2-bit heads with K = V = 128 and
// value groups of 32 (the reference's Qwen INT2 rows, quantization.py:69-87):
// signed levels {-3, -1, 1, 3} stored as (z + 3) / 2, one fp16 row scale per
// (key row, 32-value group), fp16 column scales.
//
// One 256-thread CTA per (request, 2-bit head), all modes (step, readout,
// writeback, encode, decode).  Warp w owns key rows 16w..16w+15 and lane l the
// columns l, l+32, l+64, l+96 -- so element m of a thread lies in value group
// m, and a group's 32 values of a row are element m of the warp's 32 lanes.
// Both sums of fit_state follow torch's CPU order as in the 4/6/8-bit kernels:
//  * a group's |x| sum over 32 contiguous values is 8 lanes (position % 8),
//    lane c the chain ((x_c + x_{c+8}) + x_{c+16}) + x_{c+24}, then the lanes
//    in order -- here across the warp's lanes by shuffles;
//  * the column sums over 128 rows go in 16-row blocks (one warp each), then
//    block after block.
// The step, writeback and encode keep the thread's 64 values in its
// tensor-memory lane between phases (128 columns per CTA).  Divisions by fp16
// scales use the corrected reciprocal of the other kernels (exact for such
// divisors); rows whose group |x| sum exceeds 2^96 (or is NaN) switch the tile
// to IEEE divisions.
#include "sq_fast.cuh"

namespace sq {
namespace {

constexpr int TK = 128;
constexpr int TV = 128;
constexpr int kGroup = 32;               // values per row scale
constexpr int kTwoChunk = 4;             // bytes per (row, 16-value tile): 16 codes of 2 bits
constexpr int kTwoTile = TK * kTwoChunk;  // bytes per value tile region
constexpr int kTwoCols = 128;            // tensor-memory columns per CTA

struct TwoSmem {
    uint32_t codes[8][TK + 4];  // the head's code words: value tile t, row k (16 codes), padded
    float4 rowa[TK];            // P1: {r0, r1, k, k}  P3-P5: {r0, r1, r2, r3} (the row's group scales)
    float4 rowb[TK];            // P1: {q, q, r2, r3}  P3-P5: the reciprocals of rowa
    float w2[TK];               // squared impact weights
    float red[2][8][TV];        // per-warp column partials
    float colc[4][TV];          // [0] delta, [1] c, [2] 1/c, [3] c_old * decay (c_old in decode)
    float misc[64];
    float gsum[TK][4];          // the rows' group |x| sums (P2)
    unsigned char plane[8][TK * 16 + 16];  // final codes (0..3), value tile t, row k, position u
    uint32_t tmem_slot;
};

// A thread's code of value tile t (its columns l + 32 m: t = l / 16 + 2 m) in
// row k, via the bits of the code in place: code at bit 2 u of the tile's row
// word, u = l % 16; f = 2^23 + code 2^s (s = 2 (u % 4)) from the byte, then
// 2 code = f 2^(1-s) - 2^(24-s) and z = 2 code - 3, each step exact
// (2^(24-s) + 3 itself is not a float for s = 0, so the -3 is a second add).
__device__ __forceinline__ float two_bits(const TwoSmem &s, int t, int k, int u) {
    const uint32_t w = s.codes[t][k];
    return __uint_as_float(0x4B000000u | ((w >> (8 * (u >> 2))) & (3u << (2 * (u & 3)))));
}
__device__ __forceinline__ float2 two_level_constants(int u) {
    const int sh = 2 * (u & 3);
    return make_float2(__uint_as_float(uint32_t(127 + 1 - sh) << 23), -float(1 << (24 - sh)));
}
__device__ __forceinline__ float2 two_z(float2 f, float2 lscale, float2 lbias) {
    return __fadd2_rn(pfma2(f, lscale, lbias), make_float2(-3.f, -3.f));
}

// z of fit_state's 2-bit rule: sign(y >= 0) * (|y| >= 2 ? 3 : 1).
__device__ __forceinline__ float two_level(float y) {
    const float m = fabsf(y) >= 2.f ? 3.f : 1.f;
    return y >= 0.f ? m : -m;
}

// Group |x| sums of row k in torch's order; x holds the thread's four values of
// the row (element m = group m).  Returns the sum of group (lane / 8) at lanes
// 0, 8, 16, 24 (and unused values elsewhere).
__device__ __forceinline__ float group_abs_sum(const float (&x)[4], int lane) {
    float lanes[4];
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        const float a = fabsf(x[m]);
        float b = __fadd_rn(a, __shfl_down_sync(0xffffffffu, a, 8));
        b = __fadd_rn(b, __shfl_down_sync(0xffffffffu, a, 16));
        lanes[m] = __fadd_rn(b, __shfl_down_sync(0xffffffffu, a, 24));  // lanes 0..7: chain c = lane
    }
    // lane 8 m + c takes chain c of group m, then each 8-lane segment sums in order.
    const int c = lane & 7, m = lane >> 3;
    const float g0 = __shfl_sync(0xffffffffu, lanes[0], c), g1 = __shfl_sync(0xffffffffu, lanes[1], c);
    const float g2 = __shfl_sync(0xffffffffu, lanes[2], c), g3 = __shfl_sync(0xffffffffu, lanes[3], c);
    const float v = m == 0 ? g0 : m == 1 ? g1 : m == 2 ? g2 : g3;
    float acc = v;  // (0 + chain 0) is chain 0 exactly
#pragma unroll
    for (int j = 1; j < 8; ++j) acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, v, j));
    return acc;
}

struct TwoCtx {
    int warp, lane, tid;
    uint32_t tm;
};

// P2 finish of a warp's 16 rows: the 64 group scales from the group sums in
// s.gsum, two per lane (row 16 w + lane / 2, groups 2 (lane % 2) and the next),
// into rowa (scales) and rowb (reciprocals).  Returns true for a huge or NaN
// group sum among the lane's two.
__device__ __forceinline__ bool two_row_scales(TwoSmem &s, int warp, int lane) {
    const int k = warp * 16 + (lane >> 1), m0 = 2 * (lane & 1);
    const float w = s.w2[k];
    bool huge = false;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const float total = s.gsum[k][m0 + j];
        const float mean = __fmul_rn(total, 1.f / float(kGroup));  // a power of two: the rounding of total / 32
        const float rr = fp16_scale(__fsqrt_rn(__fdiv_rn(fmaxf(mean, 1e-20f), w)));
        reinterpret_cast<float *>(&s.rowa[k])[m0 + j] = rr;
        reinterpret_cast<float *>(&s.rowb[k])[m0 + j] = __frcp_rn(rr);
        huge = huge || !(total <= 7.922816251426434e28f);  // 2^96, or NaN
    }
    return huge;
}

// P3 partial: the warp's column maxima of |x / r| -> s.red[0].  EXACT divides
// (corrected reciprocal, or IEEE on the SLOW path); otherwise the product
// x * RN(1/r), within one float step of the quotient, bounds the maximum.
template <bool SLOW, bool EXACT>
__device__ __forceinline__ void two_column_max(TwoSmem &s, const TwoCtx &c) {
    const int warp = c.warp, lane = c.lane;
    float m0 = 0.f, m1 = 0.f, m2 = 0.f, m3 = 0.f;
#pragma unroll 1
    for (int g = 0; g < 4; ++g) {
        float2 X[4][2];
        tm_ld16(c.tm + 16 * g, X);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int k = warp * 16 + 4 * g + i;
            const float4 a = s.rowa[k], b = s.rowb[k];
            const float2 s01 = EXACT ? divide2<SLOW>(X[i][0], lo2(a), lo2(b), make_float2(-a.x, -a.y)) : pmul2(X[i][0], lo2(b));
            const float2 s23 = EXACT ? divide2<SLOW>(X[i][1], hi2(a), hi2(b), make_float2(-a.z, -a.w)) : pmul2(X[i][1], hi2(b));
            m0 = fmaxf(m0, fabsf(s01.x));
            m1 = fmaxf(m1, fabsf(s01.y));
            m2 = fmaxf(m2, fabsf(s23.x));
            m3 = fmaxf(m3, fabsf(s23.y));
        }
    }
    s.red[0][warp][lane] = m0;
    s.red[0][warp][lane + 32] = m1;
    s.red[0][warp][lane + 64] = m2;
    s.red[0][warp][lane + 96] = m3;
}

// P3-P5 on the thread's values (x on entry in tensor memory; x / r on exit).
// c0 = fp16(RN(M / 3)) needs M only up to its fp16 rounding: the maximum M' of
// the products lies within one float step of M (two are allowed for), and
// when fp16(RN(. / 3)) is the same at both ends of that interval it is c0;
// otherwise the tile redoes the maxima with exact divisions.
template <bool SLOW>
__device__ __forceinline__ void two_quantize(TwoSmem &s, const TwoCtx &c) {
    const int warp = c.warp, lane = c.lane, tid = c.tid;
    two_column_max<SLOW, SLOW>(s, c);
    __syncthreads();
    int settled = 1;
    if (tid < TV) {
        float m = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) m = fmaxf(m, s.red[0][w][tid]);
        const float r3 = __frcp_rn(3.f);
        float c0;
        if (SLOW) {
            c0 = fp16_scale(__fdiv_rn(m, 3.f));
        } else {
            const uint32_t bits = __float_as_uint(m);
            const float lo = bits > 2u ? __uint_as_float(bits - 2u) : 0.f;
            c0 = fp16_scale(div_fp16(__uint_as_float(bits + 2u), 3.f, r3));
            settled = fp16_scale(div_fp16(lo, 3.f, r3)) == c0;
        }
        s.colc[1][tid] = c0;
        s.colc[2][tid] = __frcp_rn(c0);
    }
    if (!SLOW && !__syncthreads_and(settled)) {
        two_column_max<false, true>(s, c);
        __syncthreads();
        if (tid < TV) {
            float mx = 0.f;
#pragma unroll
            for (int w = 0; w < 8; ++w) mx = fmaxf(mx, s.red[0][w][tid]);
            const float c0 = fp16_scale(div_fp16(mx, 3.f, __frcp_rn(3.f)));
            s.colc[1][tid] = c0;
            s.colc[2][tid] = __frcp_rn(c0);
        }
    }
    __syncthreads();
    // P4: first levels and the weighted least-squares sums.
    {
        const float2 c01 = make_float2(s.colc[1][lane], s.colc[1][lane + 32]);
        const float2 c23 = make_float2(s.colc[1][lane + 64], s.colc[1][lane + 96]);
        const float2 r01 = make_float2(s.colc[2][lane], s.colc[2][lane + 32]);
        const float2 r23 = make_float2(s.colc[2][lane + 64], s.colc[2][lane + 96]);
        const float2 n01 = make_float2(-c01.x, -c01.y), n23 = make_float2(-c23.x, -c23.y);
        float2 num[2], den[2];
        num[0] = num[1] = den[0] = den[1] = make_float2(0.f, 0.f);
#pragma unroll 1
        for (int g = 0; g < 4; ++g) {
            float2 X[4][2];
            tm_ld16(c.tm + 16 * g, X);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int k = warp * 16 + 4 * g + i;
                const float4 a = s.rowa[k], b = s.rowb[k];
                const float2 w2 = make_float2(s.w2[k], s.w2[k]);
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const float2 rn = h ? hi2(a) : lo2(a), rr = h ? hi2(b) : lo2(b);
                    const float2 x = X[i][h];
                    const float2 sn = divide2<SLOW>(x, rn, rr, make_float2(-rn.x, -rn.y));
                    const float2 y = divide2<SLOW>(sn, h ? c23 : c01, h ? r23 : r01, h ? n23 : n01);
                    const float2 v = pmul2(rn, make_float2(two_level(y.x), two_level(y.y)));  // exact
                    num[h] = __fadd2_rn(num[h], product_term(pmul2(w2, v), x));
                    den[h] = __fadd2_rn(den[h], product_term(w2, pmul2(v, v)));
                    X[i][h] = sn;
                }
            }
            tm_st16(c.tm + 16 * g, X);
        }
        tm_wait_st();
        s.red[0][warp][lane] = num[0].x;
        s.red[0][warp][lane + 32] = num[0].y;
        s.red[0][warp][lane + 64] = num[1].x;
        s.red[0][warp][lane + 96] = num[1].y;
        s.red[1][warp][lane] = den[0].x;
        s.red[1][warp][lane + 32] = den[0].y;
        s.red[1][warp][lane + 64] = den[1].x;
        s.red[1][warp][lane + 96] = den[1].y;
    }
    __syncthreads();
    if (tid < TV) {
        float num = 0.f, den = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) {
            num = __fadd_rn(num, s.red[0][w][tid]);
            den = __fadd_rn(den, s.red[1][w][tid]);
        }
        const float c1 = den > 0.f ? fp16_scale(__fdiv_rn(num, fmaxf(den, 1e-30f))) : s.colc[1][tid];
        s.colc[1][tid] = c1;
        s.colc[2][tid] = __frcp_rn(c1);
    }
    __syncthreads();
    // P5: final levels -> code bytes (z + 3) / 2 in the plane.
    {
        const float2 c01 = make_float2(s.colc[1][lane], s.colc[1][lane + 32]);
        const float2 c23 = make_float2(s.colc[1][lane + 64], s.colc[1][lane + 96]);
        const float2 r01 = make_float2(s.colc[2][lane], s.colc[2][lane + 32]);
        const float2 r23 = make_float2(s.colc[2][lane + 64], s.colc[2][lane + 96]);
        const float2 n01 = make_float2(-c01.x, -c01.y), n23 = make_float2(-c23.x, -c23.y);
        const int t0 = lane >> 4, u = lane & 15;
#pragma unroll 1
        for (int g = 0; g < 4; ++g) {
            float2 X[4][2];
            tm_ld16(c.tm + 16 * g, X);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int k = warp * 16 + 4 * g + i;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const float2 y = divide2<SLOW>(X[i][h], h ? c23 : c01, h ? r23 : r01, h ? n23 : n01);
                    s.plane[t0 + 4 * h][k * 16 + u] = static_cast<unsigned char>((int(two_level(y.x)) + 3) >> 1);
                    s.plane[t0 + 4 * h + 2][k * 16 + u] = static_cast<unsigned char>((int(two_level(y.y)) + 3) >> 1);
                }
            }
        }
    }
    __syncthreads();
}

// Page store: code words (warp w packs its rows' chunks, four per lane), the
// rows' group scales, the column scales.
__device__ __forceinline__ void two_store(const TwoSmem &s, uint8_t *page, int off_head, int rows, int columns,
                                          const TwoCtx &c) {
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        const int i = c.lane + 32 * m, t = i >> 4, k = c.warp * 16 + (i & 15);
        const uint4 b = *reinterpret_cast<const uint4 *>(&s.plane[t][k * 16]);
        const uint32_t bytes[4] = {b.x, b.y, b.z, b.w};
        uint32_t word = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const uint32_t v = bytes[q];  // codes 4q .. 4q+3, one per byte
            word |= ((v & 3u) | ((v >> 6) & 0xCu) | ((v >> 12) & 0x30u) | ((v >> 18) & 0xC0u)) << (8 * q);
        }
        *reinterpret_cast<uint32_t *>(page + off_head + t * kTwoTile + k * kTwoChunk) = word;
    }
    if (c.lane < 16) {
        const int k = c.warp * 16 + c.lane;
        const float4 r = s.rowa[k];
        __half2 *dst = reinterpret_cast<__half2 *>(page + rows + 8 * k);  // four fp16 group scales
        dst[0] = __floats2half2_rn(r.x, r.y);
        dst[1] = __floats2half2_rn(r.z, r.w);
    }
    if (c.tid >= TK) reinterpret_cast<__half *>(page + columns)[c.tid - TK] = __float2half_rn(s.colc[1][c.tid - TK]);
}

template <int MODE>
__global__ void __launch_bounds__(kThreads) two_kernel(TileParams p, TwoHeads th) {
    // A programmatic dependent of the persistent kernel launched before it
    // (disjoint heads): its CTAs fill SMs as that kernel's CTAs leave, and each
    // waits for that kernel's completion before it exits.
    struct AfterPrimary {
        __device__ ~AfterPrimary() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
    } after_primary;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    TwoSmem &s = *reinterpret_cast<TwoSmem *>(smem_raw);
    constexpr bool kTm = MODE == kStep || MODE == kWriteback || MODE == kEncode;
    const sq_plan &P = p.plan;
    const int H = P.heads;
    TwoCtx c;
    c.tid = threadIdx.x;
    c.warp = c.tid >> 5;
    c.lane = c.tid & 31;
    const int tid = c.tid, warp = c.warp, lane = c.lane;
    const int req = blockIdx.x / th.count, head = th.ids[blockIdx.x % th.count];
    const int64_t item = int64_t(req) * H + head;
    const long long slot = p.slots[req];
    if (MODE == kReadout && head == 0 && tid == 0) p.stable_slots[req] = slot;
    if (!(slot > 0 && slot < p.num_slots)) {
        if (slot > 0 && tid == 0) flag(p.status, SQ_STATUS_SLOT_RANGE);
        if ((MODE == kStep || MODE == kReadout) && tid < TV) store_from_float(p.step.out, p.step.io_dtype, item * TV + tid, 0.f);
        if ((MODE == kStep || MODE == kDecode) && p.dense_out)
            for (int e = tid; e < TK * TV; e += kThreads) p.dense_out[item * TK * TV + e] = 0.f;
        return;
    }
    uint8_t *page = p.pages + slot * P.page_bytes;
    const int off_head = P.offsets[head * TK], rows = P.rows[head * TK], columns = P.columns[head];
    if (kTm && warp == 0) tm_alloc(&s.tmem_slot, kTwoCols);
    // ---- stage: code words, old scales, impact, inputs --------------------------
    if (MODE != kEncode) {
        for (int j = tid; j < 8 * TK; j += kThreads) s.codes[j >> 7][j & 127] = *reinterpret_cast<const uint32_t *>(page + off_head + 4 * j);
        if (tid < TK) {
            const __half2 *rw = reinterpret_cast<const __half2 *>(page + rows + 8 * tid);
            const float2 r01 = __half22float2(rw[0]);
            const float2 r23 = __half22float2(rw[1]);
            s.rowa[tid] = make_float4(r01.x, r01.y, 0.f, 0.f);
            s.rowb[tid] = make_float4(0.f, 0.f, r23.x, r23.y);
        }
        if (tid >= TK) s.colc[3][tid - TK] = half_at(page, columns + 2 * (tid - TK));
    }
    if (MODE != kReadout && MODE != kDecode && tid < TK) {
        const float w = P.impact[int64_t(head) * TK + tid];
        s.w2[tid] = w;  // (the weight itself until the row scales are taken; then its square)
    }
    float vin = 0.f, kraw = 0.f, qraw = 0.f;
    if (MODE == kStep || MODE == kReadout) {
        const sq_step_args &a = p.step;
        if (tid < TK) {
            const int qh = head / (H / a.qk_heads);
            qraw = load_as_float(a.q, a.io_dtype, int64_t(req) * a.q_stride + int64_t(qh) * TK + tid);
            kraw = load_as_float(a.k, a.io_dtype, int64_t(req) * a.k_stride + int64_t(qh) * TK + tid);
            vin = load_as_float(a.v, a.io_dtype, int64_t(req) * a.v_stride + int64_t(head) * TV + tid);
            float3 part = make_float3(__fmul_rn(qraw, qraw), __fmul_rn(kraw, kraw), __fmul_rn(qraw, kraw));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                part.x += __shfl_xor_sync(0xffffffffu, part.x, o);
                part.y += __shfl_xor_sync(0xffffffffu, part.y, o);
                part.z += __shfl_xor_sync(0xffffffffu, part.z, o);
            }
            if (lane == 0) *reinterpret_cast<float4 *>(&s.misc[4 * warp]) = make_float4(part.x, part.y, part.z, 0.f);
        }
        if (tid == kThreads - 32) {
            const float braw = load_as_float(a.beta, a.gate_dtype, item), graw = load_as_float(a.g, a.gate_dtype, item);
            const float beta = a.a_log ? 1.f / (1.f + expf(-braw)) : braw;
            float gl = graw;
            if (a.a_log) {
                const float u = gl + a.dt_bias[head];
                gl = -expf(a.a_log[head]) * (u > 20.f ? u : logf(1.f + expf(fminf(u, 20.f))));
            }
            s.misc[32] = beta;
            s.misc[33] = expf(gl);
        }
    }
    if (MODE == kWriteback && tid < TK) {
        const float *sc = p.scratch + int64_t(req) * p.scratch_stride + int64_t(head) * (TV + 2 * TK);
        s.colc[0][tid] = sc[tid];                                  // delta
        s.rowa[tid].z = s.rowa[tid].w = sc[TV + tid];               // normalised k
        if (tid == 0) s.misc[33] = sc[TV + TK];                     // decay
    }
    if (kTm) tm_fence_before();
    __syncthreads();
    if (kTm) {
        tm_fence_after();
        c.tm = s.tmem_slot + (uint32_t(32 * (warp & 3)) << 16) + uint32_t(64 * (warp >> 2));
    }
    if (MODE == kStep || MODE == kReadout) {
        // raw k and q into the row table (r_old stays in .xy / rowb.zw)
        if (tid < TK) {
            s.rowa[tid].z = s.rowa[tid].w = kraw;
            s.rowb[tid].x = s.rowb[tid].y = qraw;
        }
        __syncthreads();
    }
    if (MODE == kWriteback) {
        if (tid < TV) s.colc[3][tid] = __fmul_rn(s.colc[3][tid], s.misc[33]);  // c_old * decay
        __syncthreads();
    }

    const int t0 = lane >> 4, u = lane & 15;
    const float2 lc = two_level_constants(u);
    const float2 lscale = make_float2(lc.x, lc.x), lbias = make_float2(lc.y, lc.y);

    if (MODE == kDecode) {
        // x = (r_g c) z, as the pool's decode (fused.py codec_kernel) forms it
        const float2 c01 = make_float2(s.colc[3][lane], s.colc[3][lane + 32]);
        const float2 c23 = make_float2(s.colc[3][lane + 64], s.colc[3][lane + 96]);
        float *dst = p.dense_out + item * TK * TV;
#pragma unroll 4
        for (int r = 0; r < 16; ++r) {
            const int k = warp * 16 + r;
            const float4 a = s.rowa[k], b = s.rowb[k];
            const float2 z01 = two_z(make_float2(two_bits(s, t0, k, u), two_bits(s, t0 + 2, k, u)), lscale, lbias);
            const float2 z23 = two_z(make_float2(two_bits(s, t0 + 4, k, u), two_bits(s, t0 + 6, k, u)), lscale, lbias);
            const float2 x01 = pmul2(pmul2(lo2(a), c01), z01);
            const float2 x23 = pmul2(pmul2(hi2(b), c23), z23);
            float *row = dst + k * TV + lane;
            row[0] = x01.x;
            row[32] = x01.y;
            row[64] = x23.x;
            row[96] = x23.y;
        }
        return;
    }

    // ---- P1 (step, readout): Y = z r_old; column partials of k_raw^T Y, q_raw^T Y
    // ---- P1 + P2 (writeback): x' = Y (c_old decay) + k delta
    // ---- P1 (encode): x from the dense input
    if (MODE == kStep || MODE == kReadout) {
        float2 kx01 = make_float2(0.f, 0.f), kx23 = kx01, qx01 = kx01, qx23 = kx01;
#pragma unroll 1
        for (int g = 0; g < 4; ++g) {
            float2 X[4][2];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int k = warp * 16 + 4 * g + i;
                const float4 a = s.rowa[k], b = s.rowb[k];
                const float2 z01 = two_z(make_float2(two_bits(s, t0, k, u), two_bits(s, t0 + 2, k, u)), lscale, lbias);
                const float2 z23 = two_z(make_float2(two_bits(s, t0 + 4, k, u), two_bits(s, t0 + 6, k, u)), lscale, lbias);
                const float2 y01 = pmul2(z01, lo2(a)), y23 = pmul2(z23, hi2(b));
                X[i][0] = y01;
                X[i][1] = y23;
                kx01 = pfma2(hi2(a), y01, kx01);
                kx23 = pfma2(hi2(a), y23, kx23);
                qx01 = pfma2(lo2(b), y01, qx01);
                qx23 = pfma2(lo2(b), y23, qx23);
            }
            if (MODE == kStep) tm_st16(c.tm + 16 * g, X);
        }
        s.red[0][warp][lane] = kx01.x;
        s.red[0][warp][lane + 32] = kx01.y;
        s.red[0][warp][lane + 64] = kx23.x;
        s.red[0][warp][lane + 96] = kx23.y;
        s.red[1][warp][lane] = qx01.x;
        s.red[1][warp][lane + 32] = qx01.y;
        s.red[1][warp][lane + 64] = qx23.x;
        s.red[1][warp][lane + 96] = qx23.y;
        if (MODE == kStep) tm_wait_st();
        __syncthreads();
        if (tid < TV) {
            const sq_step_args &a = p.step;
            const float beta = s.misc[32], decay = s.misc[33];
            float qq = 0.f, kk = 0.f, dot = 0.f;
#pragma unroll
            for (int w = 0; w < TK / 32; ++w) {
                const float4 m = reinterpret_cast<const float4 *>(s.misc)[w];
                qq += m.x;
                kk += m.y;
                dot += m.z;
            }
            const float qn = a.normalize ? __frsqrt_rn(qq + 1e-6f) : 1.f;
            const float kn = a.normalize ? __frsqrt_rn(kk + 1e-6f) : 1.f;
            const float qscale = __fmul_rn(qn, a.scale);
            const float qk = __fmul_rn(__fmul_rn(__fmul_rn(dot, qn), kn), a.scale);
            float ks = 0.f, qs = 0.f;
#pragma unroll
            for (int w = 0; w < 8; ++w) {
                ks = __fadd_rn(ks, s.red[0][w][tid]);
                qs = __fadd_rn(qs, s.red[1][w][tid]);
            }
            const float cd = __fmul_rn(s.colc[3][tid], decay);
            const float kS = __fmul_rn(__fmul_rn(ks, kn), cd);
            const float qS = __fmul_rn(__fmul_rn(qs, qscale), cd);
            const float delta = __fmul_rn(beta, __fsub_rn(vin, kS));
            const float kx = __fmul_rn(kraw, kn);
            s.colc[0][tid] = delta;
            s.colc[3][tid] = cd;
            s.rowa[tid].z = kx;
            s.rowa[tid].w = kx;
            store_from_float(a.out, a.io_dtype, item * TV + tid, __fmaf_rn(qk, delta, qS));
            if (MODE == kReadout) {
                float *sc = p.scratch + int64_t(req) * p.scratch_stride + int64_t(head) * (TV + 2 * TK);
                sc[tid] = delta;
                sc[TV + tid] = kx;
                sc[TV + TK + tid] = decay;
            }
        }
        if (MODE == kReadout) return;
        __syncthreads();
    }

    // ---- P2: rank-1 update (step, writeback) or the dense input (encode); group
    // row sums -> new group scales.  A warp's rows are finished by that warp.
    bool huge = false;
    {
        const float2 d01 = make_float2(s.colc[0][lane], s.colc[0][lane + 32]);
        const float2 d23 = make_float2(s.colc[0][lane + 64], s.colc[0][lane + 96]);
        const float2 cd01 = make_float2(s.colc[3][lane], s.colc[3][lane + 32]);
        const float2 cd23 = make_float2(s.colc[3][lane + 64], s.colc[3][lane + 96]);
        float *dst = MODE == kStep && p.dense_out ? p.dense_out + item * TK * TV : nullptr;
        const float *src = MODE == kEncode ? p.dense_in + item * TK * TV : nullptr;
#pragma unroll 1
        for (int g = 0; g < 4; ++g) {
            float2 X[4][2];
            if (MODE == kStep) tm_ld16(c.tm + 16 * g, X);
            float nr[4][4];  // new values of the group's rows, element m = column lane + 32 m
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int k = warp * 16 + 4 * g + i;
                const float4 a = s.rowa[k], b = s.rowb[k];
                if (MODE == kEncode) {
                    const float *row = src + k * TV + lane;
                    X[i][0] = make_float2(row[0], row[32]);
                    X[i][1] = make_float2(row[64], row[96]);
                } else {
                    if (MODE == kWriteback) {
                        const float2 z01 = two_z(make_float2(two_bits(s, t0, k, u), two_bits(s, t0 + 2, k, u)), lscale, lbias);
                        const float2 z23 = two_z(make_float2(two_bits(s, t0 + 4, k, u), two_bits(s, t0 + 6, k, u)), lscale, lbias);
                        X[i][0] = pmul2(z01, lo2(a));
                        X[i][1] = pmul2(z23, hi2(b));
                    }
                    const float2 kk = hi2(a);
                    X[i][0] = pfma2(kk, d01, pmul2(X[i][0], cd01));
                    X[i][1] = pfma2(kk, d23, pmul2(X[i][1], cd23));
                }
                nr[i][0] = X[i][0].x;
                nr[i][1] = X[i][0].y;
                nr[i][2] = X[i][1].x;
                nr[i][3] = X[i][1].y;
                if (dst) {
                    float *row = dst + k * TV + lane;
                    row[0] = X[i][0].x;
                    row[32] = X[i][0].y;
                    row[64] = X[i][1].x;
                    row[96] = X[i][1].y;
                }
            }
            tm_st16(c.tm + 16 * g, X);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float total = group_abs_sum(nr[i], lane);
                if ((lane & 7) == 0) s.gsum[warp * 16 + 4 * g + i][lane >> 3] = total;
            }
        }
        tm_wait_st();
        __syncwarp();  // the warp's group sums are in place and its lanes are done with the old row constants
        huge = two_row_scales(s, warp, lane);
        __syncwarp();  // ... and with the unsquared weights
        if (lane < 16) {
            const int k = warp * 16 + lane;
            const float w = s.w2[k];
            s.w2[k] = __fmul_rn(w, w);
        }
    }
    const bool slow = __syncthreads_or(huge);
    if (slow) two_quantize<true>(s, c);
    else two_quantize<false>(s, c);
    two_store(s, page, off_head, rows, columns, c);
    if (kTm) {
        tm_fence_before();
        __syncthreads();
        tm_fence_after();
        if (warp == 0) tm_dealloc(s.tmem_slot, kTwoCols);
    }
}

}  // namespace

bool two_heads(const sq_plan &plan, TwoHeads *out) {
    out->count = 0;
    if (plan.architecture != SQ_GDN || plan.keys != TK || plan.values != TV || plan.storage != 0 ||
        plan.value_group_size != kGroup || !plan.bits_host)
        return false;
    for (int h = 0; h < plan.heads; ++h) {
        if (plan.bits_host[h * plan.keys] != 2) continue;
        if (out->count == kMaxTwoHeads) return false;
        out->ids[out->count++] = h;
    }
    return true;
}

cudaError_t launch_two(int mode, const TileParams &p, const TwoHeads &th, int batch, cudaStream_t stream) {
    if (th.count == 0 || batch <= 0) return cudaSuccess;
    const int grid = batch * th.count;
    constexpr int smem = int(sizeof(TwoSmem));  // below the 48 KB default limit
    static_assert(smem <= 48 * 1024, "two_kernel shared memory");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(grid));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    switch (mode) {
        case kStep: return cudaLaunchKernelEx(&cfg, two_kernel<kStep>, p, th);
        case kReadout: return cudaLaunchKernelEx(&cfg, two_kernel<kReadout>, p, th);
        case kWriteback: return cudaLaunchKernelEx(&cfg, two_kernel<kWriteback>, p, th);
        case kEncode: return cudaLaunchKernelEx(&cfg, two_kernel<kEncode>, p, th);
        case kDecode: return cudaLaunchKernelEx(&cfg, two_kernel<kDecode>, p, th);
        default: return cudaErrorNotSupported;
    }
}

}  // namespace sq
