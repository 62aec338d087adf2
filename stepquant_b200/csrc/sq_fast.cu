// Register-resident decode kernels for GDN heads with K = V = 128 and a code
// width of 4, 6 or 8 bits (the served shape of Qwen-Next-style layers).
//
// One persistent CTA per SM made of 256-thread item groups; a group
// works one (request, value head) item at a time and takes the next of its
// SM's items from a shared counter, so the groups of an SM finish together.
// The next item's page bytes and inputs are prefetched (cp.async) while the
// current item is computed.  Within a group warp w owns key rows 16w..16w+15
// and lane l owns value columns l, l+32, l+64, l+96, so each thread owns 64
// state elements for the whole step; the step, writeback and encode keep them
// in the thread's tensor-memory lane between phases and bring 16 at a time
// into registers.  That mapping makes both ordered
// sums of fit_state local:
//  * torch sums a row of 128 values as 8 lanes (column % 8), each lane a 4-way
//    interleaved chain over vectors; the chain of lane (column % 8) over the
//    columns l + 32 i is exactly what thread l holds -- only the last two
//    stages (4 partials per lane, then 8 lanes in order) cross threads;
//  * torch sums a column in 16-row blocks, then block after block; warp w's
//    16 rows are exactly block w.
// Divisions by the fp16 scales r and c use a correctly rounded reciprocal and
// one Markstein correction (q = a*y; q + (a - q*b)*y).  With a divisor of at
// most 11 significant bits a quotient cannot lie closer than 2^-12 ulp to a
// rounding midpoint, far outside the error of the corrected estimate, so the
// result equals IEEE a/b (tests/test_gpu_fast.py checks it against __fdiv_rn).
// Rows whose |x| sum exceeds 2^96 switch the CTA to IEEE divisions.
#include <algorithm>
#include <atomic>
#include <mutex>

#include <cuda.h>
#include <cudaTypedefs.h>

#include "sq_fast.cuh"

namespace sq {

namespace {

constexpr int FK = 128;
constexpr int FV = 128;
constexpr int kTile = 16;          // GDN value tile
constexpr int kTiles = FV / kTile;  // 8
constexpr int kStagePad = 16;       // bytes after each value-tile region in shared memory
constexpr int kRowPartStride = 36;  // floats per row in the row-partial exchange
constexpr int kPlaneBytes = FK * kRowPartStride * 4;  // >= kTiles * (FK * 16 + kStagePad)

template <int BITS>
struct W {
    static constexpr int chunk = 2 * BITS;           // bytes per (row, value tile): 16 codes
    static constexpr int tile_bytes = FK * chunk;    // bytes per value tile region
    static constexpr int head_bytes = tile_bytes * kTiles;
    static constexpr int off = (1 << (BITS - 1)) - 1;
};

// What one item needs from global memory, staged by cp.async one item ahead.
struct FastStage {
    unsigned char codes[kTiles * (FK * 16 + kStagePad)];  // old packed codes, padded per tile
    __half rold[FK];
    __half cold[FV];
    float in[3][FK];  // raw q, k, v (io dtype); writeback: delta, k, decay
    float imp[FK];    // the head's row impact weights
    float gate[4];    // raw beta and g (fp32 gates)
};

// Per-head constants, read once per CTA.
constexpr int kMaxHeads = 128;
struct HeadInfo {
    int width, off_head, rows, columns;
    float a_log, dt_bias;
};

// Readout and decode: the second stage buffer (the next item's data lands
// there while the current item is computed).  Step, writeback and encode: the
// row partials, then the new code bytes; these modes keep one stage buffer and
// refill it as soon as the current item's staged data has been consumed.
union FastTail {
    FastStage st1;
    unsigned char plane[kPlaneBytes];
};

// One item group's shared memory (a CTA holds kGroups of them).
struct FastSmem {
    FastStage st0;
    float red[2][8][FV];               // per-warp column partials
    float4 rowa[FK];                   // per-row constants, duplicated pairs:
    float4 rowb[FK];                   //   P1: {r_old, r_old, k, k} {q, q, -, -}; P3-P5: {r, r, 1/r, 1/r} {-r, -r, w2, w2}
    float colc[4][FV];                 // per-column constants
    float misc[64];
    HeadInfo head[kMaxHeads];
    long long slot_ring[3];  // slots of the current and next two items (cp.async)
    int item_ring[3];        // the items themselves
    uint32_t tmem_slot;      // (group 0) tensor-memory base of the CTA's columns
    alignas(16) FastTail tail;
    __device__ FastStage &stage(int b) { return b ? tail.st1 : st0; }
};

// A CTA is one SM's worth of item groups: G groups of 256 threads, each
// working one (request, head) item at a time with its own shared memory and
// named barrier, taking the SM's items one by one from a shared counter.
// Four groups at 64 registers a thread for the readout and decode; three at
// 80 for the modes that requantize (their quantizer keeps 16 state values,
// the column constants and the sums live at once).
template <int G>
struct FastCta {
    FastSmem grp[G];
    int next;  // the SM's next untaken item
};

// Barriers of one item group (ids 1..G; 0 is the CTA's __syncthreads).
__device__ __forceinline__ void group_sync(int bar) {
    asm volatile("bar.sync %0, %1;\n" ::"r"(bar), "n"(kThreads) : "memory");
}
__device__ __forceinline__ bool group_and(int bar, bool pred) {
    uint32_t r;
    asm volatile("{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, %2, %3, p;\n selp.u32 %0, 1, 0, q;\n}\n"
                 : "=r"(r) : "r"(uint32_t(pred)), "r"(bar), "n"(kThreads) : "memory");
    return r != 0;
}
__device__ __forceinline__ bool group_or(int bar, bool pred) {
    uint32_t r;
    asm volatile("{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, %2, %3, p;\n selp.u32 %0, 1, 0, q;\n}\n"
                 : "=r"(r) : "r"(uint32_t(pred)), "r"(bar), "n"(kThreads) : "memory");
    return r != 0;
}

// Step, writeback and encode keep each thread's 64 state values in tensor
// memory between phases (128 columns per item group: warps w and w + 4 share
// a lane quarter, each with 64 columns), so a thread holds only 16 of them in
// registers at a time; the four groups of a CTA take the SM's 512 columns.
template <int MODE>
__host__ __device__ constexpr bool tm_mode() { return MODE == kStep || MODE == kWriteback || MODE == kEncode; }
template <int MODE>
__host__ __device__ constexpr int groups_of() { return tm_mode<MODE>() ? 3 : 4; }

// Bits of the code of value-lane u in row k of value tile t, read from the
// staged page, ORed into the float 2^23: with the lane's conversion constants
// (level_constants) one fused multiply-add gives the exact signed level.
template <int BITS>
__device__ __forceinline__ float staged_bits(const unsigned char *stage, int t, int k, int u) {
    const unsigned char *chunk = stage + t * (W<BITS>::tile_bytes + kStagePad) + k * W<BITS>::chunk;
    uint32_t m;
    if (BITS == 8) {
        m = chunk[u];
    } else if (BITS == 4) {
        m = uint32_t(chunk[u >> 1]) & (0xFu << (4 * (u & 1)));
    } else {
        const int bit = 6 * u;
        const uint32_t w = uint32_t(chunk[bit >> 3]) | (uint32_t(chunk[(bit >> 3) + 1]) << 8);
        m = w & (0x3Fu << (bit & 7));
    }
    return __uint_as_float(0x4B000000u | m);
}

// level = bits * 2^-s - (2^(23-s) + offset), s = the code's bit shift inside the loaded unit.
template <int BITS>
__device__ __forceinline__ float2 level_constants(int u) {
    const int s = BITS == 8 ? 0 : BITS == 4 ? 4 * (u & 1) : (6 * u) & 7;
    const float scale = __uint_as_float(uint32_t(127 - s) << 23);
    return make_float2(scale, -(8388608.f * scale + float(W<BITS>::off)));
}

// Pack 16 code bytes (one per value lane) of chunk (t, k) from the plane into
// the page's 2*BITS-byte little-endian chunk.
template <int BITS>
__device__ __forceinline__ void store_chunk(uint8_t *dst, const unsigned char *plane_chunk) {
    // Plane bytes are signed levels b in [-off, off]; code = b + off per byte:
    // b ^ 0x80 = b + 128 (mod 256) lies in [128 - off, 128 + off], so
    // subtracting 128 - off from every byte never borrows across bytes.
    constexpr uint32_t sub = 0x01010101u * uint32_t(128 - W<BITS>::off);
    uint4 w = *reinterpret_cast<const uint4 *>(plane_chunk);
    w.x = (w.x ^ 0x80808080u) - sub;
    w.y = (w.y ^ 0x80808080u) - sub;
    w.z = (w.z ^ 0x80808080u) - sub;
    w.w = (w.w ^ 0x80808080u) - sub;
    if (BITS == 8) {
        *reinterpret_cast<uint4 *>(dst) = w;
    } else if (BITS == 4) {
        const uint32_t a = w.x | (w.x >> 4), b = w.y | (w.y >> 4), c = w.z | (w.z >> 4), d = w.w | (w.w >> 4);
        uint2 out;
        out.x = __byte_perm(a, b, 0x6420);
        out.y = __byte_perm(c, d, 0x6420);
        *reinterpret_cast<uint2 *>(dst) = out;
    } else {
        auto g = [](uint32_t v) {
            const uint32_t t = (v & 0x003F003Fu) | ((v >> 2) & 0x0FC00FC0u);
            return (t & 0xFFFu) | ((t >> 4) & 0xFFF000u);
        };
        const uint32_t g0 = g(w.x), g1 = g(w.y), g2 = g(w.z), g3 = g(w.w);
        uint32_t *d = reinterpret_cast<uint32_t *>(dst);
        d[0] = g0 | (g1 << 24);
        d[1] = (g1 >> 8) | (g2 << 16);
        d[2] = (g2 >> 16) | (g3 << 8);
    }
}

struct Ctx {
    int req, head, warp, lane, tid, bar;  // bar: the item group's barrier
    int64_t slot;
    uint8_t *page;
    int off_head;
    uint32_t tm;  // tensor-memory address of the thread's 64 state columns (value (4g+i, h, e) at 16g + 4i + 2h + e)
};


// P4 body: first levels z = rint(clamp(x / r / c0)) and the weighted
// least-squares numerator / denominator of the warp's 16-row block.  The
// thread's values hold x on entry and x / r on exit; rows go in groups of 4
// (one 16-column tensor-memory access), in row order.
template <bool SLOW, bool CLAMP>
__device__ __forceinline__ void first_levels(const FastSmem &s, int warp, int lane, uint32_t tm, float qmax,
                                             float2 (&num)[2], float2 (&den)[2]) {
    const float2 c01 = make_float2(s.colc[1][lane], s.colc[1][lane + 32]);
    const float2 c23 = make_float2(s.colc[1][lane + 64], s.colc[1][lane + 96]);
    const float2 r01 = make_float2(s.colc[2][lane], s.colc[2][lane + 32]);
    const float2 r23 = make_float2(s.colc[2][lane + 64], s.colc[2][lane + 96]);
    const float2 n01 = make_float2(-c01.x, -c01.y), n23 = make_float2(-c23.x, -c23.y);
    const float2 round = make_float2(kRound, kRound), nround = make_float2(-kRound, -kRound);
    num[0] = num[1] = den[0] = den[1] = make_float2(0.f, 0.f);
#pragma unroll 1
    for (int g = 0; g < 4; ++g) {
        float2 X[4][2];
        tm_ld16(tm + 16 * g, X);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float4 a = s.rowa[warp * 16 + 4 * g + i], b = s.rowb[warp * 16 + 4 * g + i];
            const float2 rn = lo2(a), w2 = hi2(b);
            // v = rn * z with z = S - 1.5*2^23: one rounding of rn*S - rn*1.5*2^23,
            // whose second product is exact (rn has 11 significant bits).
            const float2 nrk = pmul2(rn, nround);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const float2 x = X[i][h];
                const float2 sn = divide2<SLOW>(x, rn, hi2(a), lo2(b));
                float2 y = divide2<SLOW>(sn, h ? c23 : c01, h ? r23 : r01, h ? n23 : n01);
                if (CLAMP) y = clamp2(y, qmax);  // rint(clamp(y)) == clamp(rint(y)) for integer bounds
                const float2 v = pfma2(rn, __fadd2_rn(y, round), nrk);
                num[h] = __fadd2_rn(num[h], product_term(pmul2(w2, v), x));
                den[h] = __fadd2_rn(den[h], product_term(w2, pmul2(v, v)));
                X[i][h] = sn;
            }
        }
        tm_st16(tm + 16 * g, X);
    }
    tm_wait_st();
}

// P5 body: final levels -> one signed level byte per value in the plane.
template <bool SLOW, bool CLAMP>
__device__ __forceinline__ void final_levels(FastSmem &s, int warp, int lane, uint32_t tm, float qmax) {
    const float2 c01 = make_float2(s.colc[1][lane], s.colc[1][lane + 32]);
    const float2 c23 = make_float2(s.colc[1][lane + 64], s.colc[1][lane + 96]);
    const float2 r01 = make_float2(s.colc[2][lane], s.colc[2][lane + 32]);
    const float2 r23 = make_float2(s.colc[2][lane + 64], s.colc[2][lane + 96]);
    const float2 n01 = make_float2(-c01.x, -c01.y), n23 = make_float2(-c23.x, -c23.y);
    const float2 round = make_float2(kRound, kRound);
    const int t0 = lane >> 4, u = lane & 15;
    unsigned char *plane = s.tail.plane + t0 * (FK * 16 + kStagePad) + u + warp * 16 * 16;
#pragma unroll 1
    for (int g = 0; g < 4; ++g) {
        float2 X[4][2];
        tm_ld16(tm + 16 * g, X);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                float2 y = divide2<SLOW>(X[i][h], h ? c23 : c01, h ? r23 : r01, h ? n23 : n01);
                if (CLAMP) y = clamp2(y, qmax);
                const float2 code = __fadd2_rn(y, round);  // low byte: the signed level (two's complement)
                plane[(4 * h) * (FK * 16 + kStagePad) + i * 16] = static_cast<unsigned char>(__float_as_uint(code.x));
                plane[(4 * h + 2) * (FK * 16 + kStagePad) + i * 16] = static_cast<unsigned char>(__float_as_uint(code.y));
            }
        }
        plane += 4 * 16;
    }
}

// P3-P5 (shared by every width): column max -> c0; first levels and the
// weighted least-squares sums -> c1; final code bytes -> plane.  The thread's
// values (tensor memory) hold the updated state on entry and x / r on exit.
// Packed f32x2 lanes are the column pairs (l, l+32) and (l+64, l+96).  The
// clamps to [-qmax, qmax] are skipped when no level of the tile can reach
// qmax + 1/2: every |x/r| is at most the column maximum M, so
// |x/r/c| <= RN(M/c) (division and rounding are monotone).  The IEEE-division
// path (huge or NaN rows) always clamps.
// P3 partial: the warp's column maxima of |x / r| -> s.red[0].  EXACT divides
// (corrected reciprocal, or IEEE on the SLOW path); otherwise the product
// x * RN(1/r), within one ulp of the quotient, bounds the maximum.
template <bool SLOW, bool EXACT>
__device__ __forceinline__ void column_max(FastSmem &s, int warp, int lane, uint32_t tm) {
    float m0 = 0.f, m1 = 0.f, m2 = 0.f, m3 = 0.f;
#pragma unroll 1
    for (int g = 0; g < 4; ++g) {
        float2 X[4][2];
        tm_ld16(tm + 16 * g, X);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float4 a = s.rowa[warp * 16 + 4 * g + i], b = s.rowb[warp * 16 + 4 * g + i];
            const float2 s01 = EXACT ? divide2<SLOW>(X[i][0], lo2(a), hi2(a), lo2(b)) : pmul2(X[i][0], hi2(a));
            const float2 s23 = EXACT ? divide2<SLOW>(X[i][1], lo2(a), hi2(a), lo2(b)) : pmul2(X[i][1], hi2(a));
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

// P3-P5 (shared by every width): column max -> c0; first levels and the
// weighted least-squares sums -> c1; final code bytes -> plane.  The thread's
// values (tensor memory) hold the updated state on entry and x / r on exit.
// Packed f32x2 lanes are the column pairs (l, l+32) and (l+64, l+96).  The
// clamps to [-qmax, qmax] are skipped when no level of the tile can reach
// qmax + 1/2: every |x/r| is at most the column maximum M, so
// |x/r/c| <= RN(M/c) (division and rounding are monotone).  The IEEE-division
// path (huge or NaN rows) always clamps.
//
// c0 = fp16(RN(M / qmax)) needs M only up to its fp16 rounding: the maximum M'
// of the products x * RN(1/r) lies within one float step of M (two are
// allowed for), and when fp16(RN(M'' / qmax)) is the same at both ends of that
// interval it is c0 (every step is monotone).  Tiles with a column where the
// two differ redo the maxima with exact divisions.
template <bool SLOW>
__device__ __forceinline__ void fast_quantize_tail(FastSmem &s, const Ctx &c, float qmax) {
    const int warp = c.warp, lane = c.lane, tid = c.tid;
    // P3 (continued): c0 = fp16(max_k |x / r| / qmax) from the warps' partial maxima.
    int safe = 1, settled = 1;
    float mx = 0.f, ratio = 0.f, c0 = 0.f;  // mx: the exact maximum or an upper bound of it
    if (tid < FV) {
        float m = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) m = fmaxf(m, s.red[0][w][tid]);
        if (SLOW) {
            mx = m;
            ratio = __fdiv_rn(mx, qmax);
        } else {
            // qmax (7, 31 or 127) is an exact fp16 value: the corrected
            // reciprocal division is the IEEE quotient (a subnormal quotient
            // only arises below the 2^-24 clamp of fp16_scale).
            const float rq = __frcp_rn(qmax);
            const uint32_t bits = __float_as_uint(m);
            const float lo = bits > 2u ? __uint_as_float(bits - 2u) : 0.f;
            mx = __uint_as_float(bits + 2u);
            ratio = div_fp16(mx, qmax, rq);
            settled = fp16_scale(div_fp16(lo, qmax, rq)) == fp16_scale(ratio);
        }
        c0 = fp16_scale(ratio);
        s.colc[1][tid] = c0;
        s.colc[2][tid] = __frcp_rn(c0);
        // With c0 a normal, unclamped fp16 value every |x/r/c0| < qmax + 1/2.
        safe = (c0 >= 6.103515625e-05f) && (ratio <= 65504.f);
    }
    // One barrier in the common case: every column settled and safe.
    bool no_clamp = group_and(c.bar, settled && safe);
    if (!no_clamp) {
        if (!SLOW && !group_and(c.bar, settled)) {
            column_max<false, true>(s, warp, lane, c.tm);
            group_sync(c.bar);
            if (tid < FV) {
                mx = 0.f;
#pragma unroll
                for (int w = 0; w < 8; ++w) mx = fmaxf(mx, s.red[0][w][tid]);
                ratio = __fdiv_rn(mx, qmax);
                c0 = fp16_scale(ratio);
                s.colc[1][tid] = c0;
                s.colc[2][tid] = __frcp_rn(c0);
                safe = (c0 >= 6.103515625e-05f) && (ratio <= 65504.f);
            }
        }
        no_clamp = group_and(c.bar, safe);
    }
    // P4: first levels, weighted least-squares numerator / denominator (16-row blocks).
    {
        float2 num[2], den[2];
        if (!SLOW && no_clamp) first_levels<SLOW, false>(s, warp, lane, c.tm, qmax, num, den);
        else first_levels<SLOW, true>(s, warp, lane, c.tm, qmax, num, den);
        s.red[0][warp][lane] = num[0].x;
        s.red[0][warp][lane + 32] = num[0].y;
        s.red[0][warp][lane + 64] = num[1].x;
        s.red[0][warp][lane + 96] = num[1].y;
        s.red[1][warp][lane] = den[0].x;
        s.red[1][warp][lane + 32] = den[0].y;
        s.red[1][warp][lane + 64] = den[1].x;
        s.red[1][warp][lane + 96] = den[1].y;
    }
    group_sync(c.bar);
    safe = 1;
    if (tid < FV) {
        float num = 0.f, den = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) {
            num = __fadd_rn(num, s.red[0][w][tid]);
            den = __fadd_rn(den, s.red[1][w][tid]);
        }
        const float c1 = den > 0.f ? fp16_scale(__fdiv_rn(num, fmaxf(den, 1e-30f))) : s.colc[1][tid];
        const float rc1 = __frcp_rn(c1);
        s.colc[1][tid] = c1;
        s.colc[2][tid] = rc1;
        // (an overflowing quotient reads as unsafe; an underflowing one is far below qmax)
        safe = (c1 >= 6.103515625e-05f) && ((SLOW ? __fdiv_rn(mx, c1) : div_fp16(mx, c1, rc1)) < qmax + 0.5f);
    }
    const bool no_clamp5 = group_and(c.bar, safe);
    // P5: final levels -> one signed level byte per value in the plane.
    if (!SLOW && no_clamp5) final_levels<SLOW, false>(s, warp, lane, c.tm, qmax);
    else final_levels<SLOW, true>(s, warp, lane, c.tm, qmax);
    // Every code byte of a row comes from the warp that owns the row, and that
    // warp packs the row's chunks (fast_store).
    __syncwarp();
}

// P3-P5.  `warp_slow`: a row of this warp has an |x| sum beyond 2^96 (or NaN),
// so its partial maxima use IEEE divisions; the whole tile switches to IEEE
// divisions when any warp is slow (the partial maxima of the other warps are
// then taken again with IEEE divisions).  The barrier that completes the
// partial maxima also combines the warps' flags.
// `consumed` runs right after that barrier, when every thread of the group is
// past its last read of the item's stage buffer.
template <class Consumed>
__device__ __forceinline__ void fast_quantize(FastSmem &s, const Ctx &c, float qmax, bool warp_slow, Consumed &&consumed) {
    if (warp_slow) column_max<true, true>(s, c.warp, c.lane, c.tm);
    else column_max<false, false>(s, c.warp, c.lane, c.tm);
    const bool slow = group_or(c.bar, warp_slow);
    consumed();
    if (slow) {
        if (!warp_slow) column_max<true, true>(s, c.warp, c.lane, c.tm);
        group_sync(c.bar);
        fast_quantize_tail<true>(s, c, qmax);
    } else {
        fast_quantize_tail<false>(s, c, qmax);
    }
}

// Pack the code plane into the page (2*BITS bytes per row-tile chunk) and store r and c.
// Warp w packs the chunks of its own rows 16w..16w+15 (all eight value tiles),
// four per lane, and stores their row scales; threads 128-255 store c.
template <int BITS>
__device__ __forceinline__ void fast_store(FastSmem &s, const Ctx &c) {
    uint8_t *dst = c.page + c.off_head;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        const int i = c.lane + 32 * m, t = i >> 4, k = c.warp * 16 + (i & 15);
        store_chunk<BITS>(dst + t * W<BITS>::tile_bytes + k * W<BITS>::chunk, s.tail.plane + t * (FK * 16 + kStagePad) + k * 16);
    }
    const HeadInfo &hi = s.head[c.head];
    if (c.lane < 16) {
        const int k = c.warp * 16 + c.lane;
        reinterpret_cast<__half *>(c.page + hi.rows)[k] = __float2half_rn(s.rowa[k].x);
    }
    if (c.tid >= FK) reinterpret_cast<__half *>(c.page + hi.columns)[c.tid - FK] = __float2half_rn(s.colc[1][c.tid - FK]);
}

// Stage the head's code bytes (cp.async, 16-byte pieces, one padded region per value tile).
template <int BITS>
__device__ __forceinline__ void stage_codes(FastStage &st, const uint8_t *src, int tid) {
    constexpr int pieces = W<BITS>::head_bytes / 16;
    constexpr int per_tile = W<BITS>::tile_bytes / 16;
    for (int j = tid; j < pieces; j += kThreads) {
        const int t = j / per_tile, within = j % per_tile;
        cp_async16(st.codes + t * (W<BITS>::tile_bytes + kStagePad) + within * 16, src + j * 16);
    }
}

// P1 of the readout, which keeps no state: the column partials of k_raw^T Y
// and q_raw^T Y, with lane l covering the four consecutive columns 4l..4l+3
// (one or two word loads per row instead of a byte load per value).  Each
// column's partial is the same ordered sum over the warp's 16 rows as in
// unpack_rows_tm, so the results are identical.
template <int BITS>
__device__ __forceinline__ void readout_rows(FastSmem &s, const FastStage &st, int warp, int lane) {
    const int gq = lane & 3;
    const unsigned char *tile = st.codes + (lane >> 2) * (W<BITS>::tile_bytes + kStagePad);
    constexpr float off = float(W<BITS>::off);
    // Code i of the lane's four is taken with its bits in place, ORed into
    // 2^23; level = f * 2^-(its bit position) - (2^(23 - position) + offset),
    // exact (8-bit codes are moved to bit 0 by a byte permute; the fourth 6-bit
    // code by a shift, its bits would reach the exponent field).
    constexpr int p1 = BITS == 8 ? 0 : BITS, p2 = BITS == 8 ? 0 : 2 * BITS, p3 = BITS == 4 ? 12 : 0;
    const float2 sc01 = make_float2(1.f, __uint_as_float(uint32_t(127 - p1) << 23));
    const float2 sc23 = make_float2(__uint_as_float(uint32_t(127 - p2) << 23), __uint_as_float(uint32_t(127 - p3) << 23));
    const float2 bi01 = make_float2(-(8388608.f + off), -(8388608.f * sc01.y + off));
    const float2 bi23 = make_float2(-(8388608.f * sc23.x + off), -(8388608.f * sc23.y + off));
    float2 kx01 = make_float2(0.f, 0.f), kx23 = kx01, qx01 = kx01, qx23 = kx01;
#pragma unroll 4
    for (int r = 0; r < 16; ++r) {
        const int k = warp * 16 + r;
        const unsigned char *chunk = tile + k * W<BITS>::chunk;
        uint32_t f0, f1, f2, f3;
        if (BITS == 8) {
            const uint32_t v = *reinterpret_cast<const uint32_t *>(chunk + 4 * gq);
            f0 = __byte_perm(v, 0x4B000000u, 0x7650);
            f1 = __byte_perm(v, 0x4B000000u, 0x7651);
            f2 = __byte_perm(v, 0x4B000000u, 0x7652);
            f3 = __byte_perm(v, 0x4B000000u, 0x7653);
        } else if (BITS == 4) {
            const uint32_t v = *reinterpret_cast<const uint16_t *>(chunk + 2 * gq);
            f0 = 0x4B000000u | (v & 0xFu);
            f1 = 0x4B000000u | (v & 0xF0u);
            f2 = 0x4B000000u | (v & 0xF00u);
            f3 = 0x4B000000u | (v & 0xF000u);
        } else {  // 3 bytes at 3 gq: two words and a funnel shift (the second word may be the next chunk's)
            const uint32_t *words = reinterpret_cast<const uint32_t *>(chunk) + ((3 * gq) >> 2);
            const uint32_t v = __funnelshift_r(words[0], words[1], (3 * gq & 3) * 8);
            f0 = 0x4B000000u | (v & 0x3Fu);
            f1 = 0x4B000000u | (v & 0xFC0u);
            f2 = 0x4B000000u | (v & 0x3F000u);
            f3 = 0x4B000000u | ((v >> 18) & 0x3Fu);
        }
        const float4 a = s.rowa[k], b = s.rowb[k];
        const float2 y01 = pmul2(pfma2(make_float2(__uint_as_float(f0), __uint_as_float(f1)), sc01, bi01), lo2(a));
        const float2 y23 = pmul2(pfma2(make_float2(__uint_as_float(f2), __uint_as_float(f3)), sc23, bi23), lo2(a));
        kx01 = pfma2(hi2(a), y01, kx01);
        kx23 = pfma2(hi2(a), y23, kx23);
        qx01 = pfma2(lo2(b), y01, qx01);
        qx23 = pfma2(lo2(b), y23, qx23);
    }
    *reinterpret_cast<float4 *>(&s.red[0][warp][4 * lane]) = make_float4(kx01.x, kx01.y, kx23.x, kx23.y);
    *reinterpret_cast<float4 *>(&s.red[1][warp][4 * lane]) = make_float4(qx01.x, qx01.y, qx23.x, qx23.y);
}

// P1 of the fused step: unpack the warp's 16 rows into Y = level * r_old
// (to tensor memory) and accumulate the column partials of k_raw^T Y and
// q_raw^T Y.
template <int BITS>
__device__ __forceinline__ void unpack_rows_tm(const FastSmem &s, const FastStage &st, int warp, int lane, uint32_t tm,
                                               float2 (&acc)[4]) {
    const int t0 = lane >> 4, u = lane & 15;
    const float2 lc = level_constants<BITS>(u);
    const float2 lscale = make_float2(lc.x, lc.x), lbias = make_float2(lc.y, lc.y);
    float2 kx01 = make_float2(0.f, 0.f), kx23 = kx01, qx01 = kx01, qx23 = kx01;
#pragma unroll 1
    for (int g = 0; g < 4; ++g) {
        float2 X[4][2];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int k = warp * 16 + 4 * g + i;
            const float4 a = s.rowa[k], b = s.rowb[k];
            const float2 f01 = make_float2(staged_bits<BITS>(st.codes, t0, k, u), staged_bits<BITS>(st.codes, t0 + 2, k, u));
            const float2 f23 = make_float2(staged_bits<BITS>(st.codes, t0 + 4, k, u), staged_bits<BITS>(st.codes, t0 + 6, k, u));
            const float2 x01 = pmul2(pfma2(f01, lscale, lbias), lo2(a));
            const float2 x23 = pmul2(pfma2(f23, lscale, lbias), lo2(a));
            X[i][0] = x01;
            X[i][1] = x23;
            kx01 = pfma2(hi2(a), x01, kx01);
            kx23 = pfma2(hi2(a), x23, kx23);
            qx01 = pfma2(lo2(b), x01, qx01);
            qx23 = pfma2(lo2(b), x23, qx23);
        }
        tm_st16(tm + 16 * g, X);
    }
    acc[0] = kx01;
    acc[1] = kx23;
    acc[2] = qx01;
    acc[3] = qx23;
}

// Row |x| partial of row k in torch's order: one thread's 4 columns l, l+32,
// l+64, l+96 are one accumulator slot of the 8-lane, 4-way interleaved chain.
__device__ __forceinline__ void row_partial(float *rowpart, int k, int lane, const float2 (&x)[2]) {
    // (0 + |x0|) + |x1| + ... in torch's order; 0 + |x0| is |x0| exactly.
    rowpart[k * kRowPartStride + lane] =
        __fadd_rn(__fadd_rn(__fadd_rn(fabsf(x[0].x), fabsf(x[0].y)), fabsf(x[1].x)), fabsf(x[1].y));
}

// P1 + P2 of the writeback (delta, k and c * decay are known before the
// unpack): x' = (level * r_old) * (c * decay) + k * delta, row partials, x' to
// tensor memory.
template <int BITS>
__device__ __forceinline__ void unpack_update_tm(FastSmem &s, const FastStage &st, int warp, int lane, uint32_t tm) {
    const int t0 = lane >> 4, u = lane & 15;
    const float2 lc = level_constants<BITS>(u);
    const float2 lscale = make_float2(lc.x, lc.x), lbias = make_float2(lc.y, lc.y);
    const float2 d01 = make_float2(s.colc[0][lane], s.colc[0][lane + 32]);
    const float2 d23 = make_float2(s.colc[0][lane + 64], s.colc[0][lane + 96]);
    const float2 cd01 = make_float2(s.colc[3][lane], s.colc[3][lane + 32]);
    const float2 cd23 = make_float2(s.colc[3][lane + 64], s.colc[3][lane + 96]);
    float *rowpart = reinterpret_cast<float *>(s.tail.plane);
#pragma unroll 1
    for (int g = 0; g < 4; ++g) {
        float2 X[4][2];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int k = warp * 16 + 4 * g + i;
            const float4 a = s.rowa[k];
            const float2 f01 = make_float2(staged_bits<BITS>(st.codes, t0, k, u), staged_bits<BITS>(st.codes, t0 + 2, k, u));
            const float2 f23 = make_float2(staged_bits<BITS>(st.codes, t0 + 4, k, u), staged_bits<BITS>(st.codes, t0 + 6, k, u));
            const float2 x01 = pmul2(pfma2(f01, lscale, lbias), lo2(a));
            const float2 x23 = pmul2(pfma2(f23, lscale, lbias), lo2(a));
            X[i][0] = pfma2(hi2(a), d01, pmul2(x01, cd01));
            X[i][1] = pfma2(hi2(a), d23, pmul2(x23, cd23));
            row_partial(rowpart, k, lane, X[i]);
        }
        tm_st16(tm + 16 * g, X);
    }
}

// P1 + P2 of the encode: the dense state rows, row partials, to tensor memory.
__device__ __forceinline__ void load_rows_tm(FastSmem &s, const float *src, int warp, int lane, uint32_t tm) {
    float *rowpart = reinterpret_cast<float *>(s.tail.plane);
#pragma unroll 1
    for (int g = 0; g < 4; ++g) {
        float2 X[4][2];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int k = warp * 16 + 4 * g + i;
            const float *row = src + k * FV + lane;
            X[i][0] = make_float2(row[0], row[32]);
            X[i][1] = make_float2(row[64], row[96]);
            row_partial(rowpart, k, lane, X[i]);
        }
        tm_st16(tm + 16 * g, X);
    }
}

// Decode of one width: x = (r * c) * level (the order of the reference codec),
// written to the dense output.
template <int BITS>
__device__ __forceinline__ void decode_rows(const FastStage &st, int warp, int lane, float *dst) {
    const int t0 = lane >> 4, u = lane & 15;
    const float2 c01 = make_float2(__half2float(st.cold[lane]), __half2float(st.cold[lane + 32]));
    const float2 c23 = make_float2(__half2float(st.cold[lane + 64]), __half2float(st.cold[lane + 96]));
    const float2 lc = level_constants<BITS>(u);
    const float2 lscale = make_float2(lc.x, lc.x), lbias = make_float2(lc.y, lc.y);
#pragma unroll
    for (int r = 0; r < 16; ++r) {
        const int k = warp * 16 + r;
        const float rk = __half2float(st.rold[k]);
        const float2 rr = make_float2(rk, rk);
        const float2 f01 = make_float2(staged_bits<BITS>(st.codes, t0, k, u), staged_bits<BITS>(st.codes, t0 + 2, k, u));
        const float2 f23 = make_float2(staged_bits<BITS>(st.codes, t0 + 4, k, u), staged_bits<BITS>(st.codes, t0 + 6, k, u));
        const float2 x01 = pmul2(pmul2(rr, c01), pfma2(f01, lscale, lbias));
        const float2 x23 = pmul2(pmul2(rr, c23), pfma2(f23, lscale, lbias));
        float *row = dst + k * FV + lane;
        row[0] = x01.x;
        row[32] = x01.y;
        row[64] = x23.x;
        row[96] = x23.y;
    }
}

// fp16 pivot heads (width 16): the page holds x.half() of every value in the
// value-tile layout -- tile t (16 values) is 128 rows of 32 bytes -- and no
// scales.  Lane l covers the four consecutive columns 4l..4l+3 (tile l / 4,
// bytes 8 (l % 4) .. +7 of a row), warp w the rows 16w..16w+15; a pivot head
// is read straight from global memory (it is not staged).
__device__ __forceinline__ uint8_t *pivot_lane(uint8_t *head, int warp, int lane) {
    return head + (lane >> 2) * (FK * 32) + (lane & 3) * 8 + warp * 16 * 32;
}
__device__ __forceinline__ void halves4(uint2 raw, float2 &lo, float2 &hi) {
    lo = __half22float2(*reinterpret_cast<const __half2 *>(&raw.x));
    hi = __half22float2(*reinterpret_cast<const __half2 *>(&raw.y));
}

// The pivot head's two passes on the warp's 16 rows, held in registers (the
// pivot kernel loads them once, ahead of its inputs): the column partials of
// k_raw^T Y and q_raw^T Y over the rows in order (as readout_rows), then the
// update in place, x' = Y (c decay) + k delta per value (the same operations
// as the integer heads' update) stored as fp16, the fp32 x' also to `dense`
// ([K, V] of this item) when given.
template <class Smem>
__device__ __forceinline__ void pivot_rows_held(Smem &s, const uint2 (&raw)[16], int warp, int lane) {
    float2 kx01 = make_float2(0.f, 0.f), kx23 = kx01, qx01 = kx01, qx23 = kx01;
#pragma unroll
    for (int r = 0; r < 16; ++r) {
        const int k = warp * 16 + r;
        float2 y01, y23;
        halves4(raw[r], y01, y23);
        const float4 a = s.rowa[k], b = s.rowb[k];
        kx01 = pfma2(hi2(a), y01, kx01);
        kx23 = pfma2(hi2(a), y23, kx23);
        qx01 = pfma2(lo2(b), y01, qx01);
        qx23 = pfma2(lo2(b), y23, qx23);
    }
    *reinterpret_cast<float4 *>(&s.red[0][warp][4 * lane]) = make_float4(kx01.x, kx01.y, kx23.x, kx23.y);
    *reinterpret_cast<float4 *>(&s.red[1][warp][4 * lane]) = make_float4(qx01.x, qx01.y, qx23.x, qx23.y);
}

template <class Smem>
__device__ __forceinline__ void pivot_update_held(const Smem &s, const uint2 (&raw)[16], uint8_t *head, int warp,
                                                  int lane, float *dense) {
    uint8_t *dst = pivot_lane(head, warp, lane);
    const float4 d = *reinterpret_cast<const float4 *>(&s.colc[0][4 * lane]);
    const float4 cd = *reinterpret_cast<const float4 *>(&s.colc[3][4 * lane]);
    const float2 d01 = lo2(d), d23 = hi2(d), cd01 = lo2(cd), cd23 = hi2(cd);
#pragma unroll
    for (int r = 0; r < 16; ++r) {
        const int k = warp * 16 + r;
        float2 y01, y23;
        halves4(raw[r], y01, y23);
        const float2 kk = hi2(s.rowa[k]);
        const float2 x01 = pfma2(kk, d01, pmul2(y01, cd01));
        const float2 x23 = pfma2(kk, d23, pmul2(y23, cd23));
        const __half2 h01 = __float22half2_rn(x01), h23 = __float22half2_rn(x23);
        *reinterpret_cast<uint2 *>(dst + r * 32) =
            make_uint2(*reinterpret_cast<const uint32_t *>(&h01), *reinterpret_cast<const uint32_t *>(&h23));
        if (dense) *reinterpret_cast<float4 *>(dense + k * FV + 4 * lane) = make_float4(x01.x, x01.y, x23.x, x23.y);
    }
}

// Encode / decode of a pivot head: dense fp32 rows <-> fp16 values.
__device__ __forceinline__ void pivot_encode(const float *src, uint8_t *head, int warp, int lane) {
    uint8_t *dst = pivot_lane(head, warp, lane);
#pragma unroll
    for (int r = 0; r < 16; ++r) {
        const float4 x = *reinterpret_cast<const float4 *>(src + (warp * 16 + r) * FV + 4 * lane);
        const __half2 h01 = __floats2half2_rn(x.x, x.y), h23 = __floats2half2_rn(x.z, x.w);
        *reinterpret_cast<uint2 *>(dst + r * 32) =
            make_uint2(*reinterpret_cast<const uint32_t *>(&h01), *reinterpret_cast<const uint32_t *>(&h23));
    }
}
__device__ __forceinline__ void pivot_decode(uint8_t *head, float *dst, int warp, int lane) {
    const uint8_t *src = pivot_lane(head, warp, lane);
#pragma unroll
    for (int r = 0; r < 16; ++r) {
        float2 y01, y23;
        halves4(*reinterpret_cast<const uint2 *>(src + r * 32), y01, y23);
        *reinterpret_cast<float4 *>(dst + (warp * 16 + r) * FV + 4 * lane) = make_float4(y01.x, y01.y, y23.x, y23.y);
    }
}

// One (request, head) work item of the persistent loop.
struct WorkItem {
    int req, head, width;
    int64_t slot;
    bool fast;    // code width handled by these kernels (else the tile kernel's)
    bool active;  // 0 < slot < num_slots
};

__device__ __forceinline__ WorkItem describe(const TileParams &p, const FastSmem &s, int req, int head, long long slot) {
    WorkItem it;
    it.req = req;
    it.head = head;
    it.slot = slot;
    it.width = s.head[it.head].width;
    it.fast = it.width == 4 || it.width == 6 || it.width == 8;
    it.active = it.slot > 0 && it.slot < p.num_slots;
    return it;
}

// Issue the cp.async copies of everything item `it` reads: its code bytes, the
// old r and c, and (when the host found them 16-byte aligned) the request's
// q, k, v and fp32 gates, or for the writeback the readout's delta, k and decay.
// Threads 0-31 copy r and c, 32-127 the inputs, 128-129 the gates, 160-191
// the impact row.
template <int MODE>
__device__ __forceinline__ void prefetch(const TileParams &p, const FastSmem &s, FastStage &st, const WorkItem &it, int tid) {
    const sq_plan &P = p.plan;
    const HeadInfo &hi = s.head[it.head];
    const uint8_t *page = p.pages + it.slot * P.page_bytes;
    const uint8_t *src = page + hi.off_head;
    if (MODE != kEncode) {
        if (it.width == 4) stage_codes<4>(st, src, tid);
        else if (it.width == 6) stage_codes<6>(st, src, tid);
        else stage_codes<8>(st, src, tid);
        if (tid < 16) cp_async16(reinterpret_cast<unsigned char *>(st.rold) + tid * 16, page + hi.rows + tid * 16);
        else if (tid < 32) cp_async16(reinterpret_cast<unsigned char *>(st.cold) + (tid - 16) * 16, page + hi.columns + (tid - 16) * 16);
    }
    if (MODE != kReadout && MODE != kDecode && tid >= 160 && tid < 192)
        cp_async16(reinterpret_cast<unsigned char *>(st.imp) + (tid - 160) * 16, P.impact + int64_t(it.head) * FK + (tid - 160) * 4);
    if (MODE == kEncode || MODE == kDecode || !p.stage_inputs) return;
    unsigned char *in = reinterpret_cast<unsigned char *>(st.in);
    const int j = tid - 32;
    if (MODE == kWriteback) {
        // delta[V], k[K], decay: 65 pieces of the request's scratch row.
        const float *sc = p.scratch + int64_t(it.req) * p.scratch_stride + int64_t(it.head) * (FV + 2 * FK);
        if (j >= 0 && j < 65) cp_async16(in + j * 16, sc + j * 4);
    } else {
        const sq_step_args &a = p.step;
        const int esize = a.io_dtype == SQ_F32 ? 4 : 2;
        const int pshift = esize == 4 ? 5 : 4;  // 16-byte pieces per row: FK * esize / 16
        if (j >= 0 && j < (3 << pshift)) {
            const int which = j >> pshift, piece = j & ((1 << pshift) - 1);
            const int qh = it.head / (P.heads / a.qk_heads);
            const unsigned char *base =
                which == 0 ? static_cast<const unsigned char *>(a.q) + (int64_t(it.req) * a.q_stride + int64_t(qh) * FK) * esize
                : which == 1 ? static_cast<const unsigned char *>(a.k) + (int64_t(it.req) * a.k_stride + int64_t(qh) * FK) * esize
                             : static_cast<const unsigned char *>(a.v) + (int64_t(it.req) * a.v_stride + int64_t(it.head) * FV) * esize;
            cp_async16(in + which * (FK * 4) + piece * 16, base + piece * 16);
        }
        if (p.stage_gates) {
            const int64_t g = int64_t(it.req) * P.heads + it.head;
            if (tid == 128) cp_async4(&st.gate[0], static_cast<const float *>(a.beta) + g);
            else if (tid == 129) cp_async4(&st.gate[1], static_cast<const float *>(a.g) + g);
        }
    }
}

// ---------------------------------------------------------------------------
// The per-head body.  MODE: kStep (fused), kReadout, kWriteback.  Only the
// staging, unpack and pack steps depend on the code width; the prologue, the
// update and the quantizer are one copy shared by every width, so CTAs of
// different widths resident on one SM run the same instructions.
// ---------------------------------------------------------------------------
template <int MODE, class Consumed>
__device__ void fast_body(const TileParams &p, FastSmem &s, const FastStage &st, const Ctx &c, int width,
                          Consumed &&consumed) {
    const sq_plan &P = p.plan;
    const int H = P.heads;
    const int warp = c.warp, lane = c.lane, tid = c.tid;
    if (MODE == kDecode) {
        float *dst = p.dense_out + (int64_t(c.req) * H + c.head) * FK * FV;
        if (width == 4) decode_rows<4>(st, warp, lane, dst);
        else if (width == 6) decode_rows<6>(st, warp, lane, dst);
        else decode_rows<8>(st, warp, lane, dst);
        return;
    }

    // ---- per-request inputs -------------------------------------------------
    // P1 works on Y = level * r_old (no decay, no column scale) with raw q and
    // k, so it needs nothing computed here: the gate and norm chains overlap
    // with the unpack.  The updated state is x' = Y * (c * decay) + k * delta,
    // and k^T (D S) = kn * (c * decay) * sum_k(k_raw * Y) (likewise for q).
    float vin = 0.f, kraw = 0.f, braw = 0.f, graw = 0.f;
    if (MODE == kEncode) {
        // nothing: the state comes from the dense input
    } else if (MODE == kWriteback) {
        const float *sc = p.scratch + int64_t(c.req) * p.scratch_stride + int64_t(c.head) * (FV + 2 * FK);
        if (tid < FK) {
            const float delta = p.stage_inputs ? st.in[0][tid] : sc[tid];
            const float kx = p.stage_inputs ? st.in[1][tid] : sc[FV + tid];  // normalised k
            const float decay = p.stage_inputs ? st.in[2][0] : sc[FV + FK];
            const float ro = __half2float(st.rold[tid]);
            s.rowa[tid] = make_float4(ro, ro, kx, kx);
            s.colc[0][tid] = delta;
            s.colc[3][tid] = __fmul_rn(__half2float(st.cold[tid]), decay);
        }
    } else {
        const sq_step_args &a = p.step;
        float qraw = 0.f;
        if (tid < FK) {
            if (p.stage_inputs) {
                qraw = load_as_float(st.in[0], a.io_dtype, tid);
                kraw = load_as_float(st.in[1], a.io_dtype, tid);
                vin = load_as_float(st.in[2], a.io_dtype, tid);
            } else {
                const int qh = c.head / (H / a.qk_heads);
                qraw = load_as_float(a.q, a.io_dtype, int64_t(c.req) * a.q_stride + int64_t(qh) * FK + tid);
                kraw = load_as_float(a.k, a.io_dtype, int64_t(c.req) * a.k_stride + int64_t(qh) * FK + tid);
                vin = load_as_float(a.v, a.io_dtype, int64_t(c.req) * a.v_stride + int64_t(c.head) * FV + tid);
            }
            const float ro = __half2float(st.rold[tid]);
            s.rowa[tid] = make_float4(ro, ro, kraw, kraw);
            s.rowb[tid] = make_float4(qraw, qraw, 0.f, 0.f);
        }
        if (tid == kThreads - 32) {
            // The item's two gates, once, by a thread of the last warp (idle
            // here): beta = sigmoid(b), decay = exp(-exp(A_log) softplus(a + dt_bias)).
            braw = p.stage_gates ? st.gate[0] : load_as_float(a.beta, a.gate_dtype, int64_t(c.req) * H + c.head);
            graw = p.stage_gates ? st.gate[1] : load_as_float(a.g, a.gate_dtype, int64_t(c.req) * H + c.head);
            const float beta = a.a_log ? 1.f / (1.f + expf(-braw)) : braw;
            float g = graw;
            if (a.a_log) {
                const float u = g + s.head[c.head].dt_bias;
                g = -expf(s.head[c.head].a_log) * (u > 20.f ? u : logf(1.f + expf(fminf(u, 20.f))));
            }
            s.misc[32] = beta;
            s.misc[33] = expf(g);
        }
        // Per-warp sums of q^2, k^2 and q.k over the warps holding q and k
        // (threads 0..K-1), combined after the next barrier.
        if (tid < FK) {
            float3 part = make_float3(__fmul_rn(qraw, qraw), __fmul_rn(kraw, kraw), __fmul_rn(qraw, kraw));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                part.x += __shfl_xor_sync(0xffffffffu, part.x, o);
                part.y += __shfl_xor_sync(0xffffffffu, part.y, o);
                part.z += __shfl_xor_sync(0xffffffffu, part.z, o);
            }
            if (lane == 0) *reinterpret_cast<float4 *>(&s.misc[4 * warp]) = make_float4(part.x, part.y, part.z, 0.f);
        }
    }
    group_sync(c.bar);

    // ---- P1: unpack; column partials of k_raw^T Y and q_raw^T Y ---------------
    // (Encode and writeback fold P2's work into this pass.)
    if (MODE == kEncode) {
        load_rows_tm(s, p.dense_in + (int64_t(c.req) * H + c.head) * FK * FV, warp, lane, c.tm);
    } else if (MODE == kWriteback) {
        if (width == 4) unpack_update_tm<4>(s, st, warp, lane, c.tm);
        else if (width == 6) unpack_update_tm<6>(s, st, warp, lane, c.tm);
        else unpack_update_tm<8>(s, st, warp, lane, c.tm);
    } else {
        if (MODE == kReadout) {
            if (width == 4) readout_rows<4>(s, st, warp, lane);
            else if (width == 6) readout_rows<6>(s, st, warp, lane);
            else readout_rows<8>(s, st, warp, lane);
        } else {
            float2 acc[4];
            if (width == 4) unpack_rows_tm<4>(s, st, warp, lane, c.tm, acc);
            else if (width == 6) unpack_rows_tm<6>(s, st, warp, lane, c.tm, acc);
            else unpack_rows_tm<8>(s, st, warp, lane, c.tm, acc);
            s.red[0][warp][lane] = acc[0].x;
            s.red[0][warp][lane + 32] = acc[0].y;
            s.red[0][warp][lane + 64] = acc[1].x;
            s.red[0][warp][lane + 96] = acc[1].y;
            s.red[1][warp][lane] = acc[2].x;
            s.red[1][warp][lane + 32] = acc[2].y;
            s.red[1][warp][lane + 64] = acc[3].x;
            s.red[1][warp][lane + 96] = acc[3].y;
        }
        {
            const sq_step_args &a = p.step;
            // Norms and the column results: the four warps of the value columns.
            group_sync(c.bar);
            if (tid < FV) {
                const float beta = s.misc[32], decay = s.misc[33];
                float qq = 0.f, kk = 0.f, dot = 0.f;
#pragma unroll
                for (int w = 0; w < FK / 32; ++w) {
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
                const float cd = __fmul_rn(__half2float(st.cold[tid]), decay);
                const float kS = __fmul_rn(__fmul_rn(ks, kn), cd);      // k^T (D S)
                const float qS = __fmul_rn(__fmul_rn(qs, qscale), cd);  // q^T (D S)
                const float delta = __fmul_rn(beta, __fsub_rn(vin, kS));
                const float kx = __fmul_rn(kraw, kn);  // row tid of the normalised k
                s.colc[0][tid] = delta;
                s.colc[3][tid] = cd;
                s.rowa[tid].z = kx;
                s.rowa[tid].w = kx;
                store_from_float(a.out, a.io_dtype, (int64_t(c.req) * H + c.head) * FV + tid, __fmaf_rn(qk, delta, qS));
                if (MODE == kReadout) {
                    float *sc = p.scratch + int64_t(c.req) * p.scratch_stride + int64_t(c.head) * (FV + 2 * FK);
                    sc[tid] = delta;
                    sc[FV + tid] = kx;
                    sc[FV + FK + tid] = decay;
                }
            }
            if (MODE == kReadout) return;
            group_sync(c.bar);
        }
    }

    // ---- P2: rank-1 update; row sums of |x| in torch order; new row scales ---
    bool warp_slow;
    {
        bool huge = false;
        float *rowpart = reinterpret_cast<float *>(s.tail.plane);
        if (MODE == kStep) {
            const float2 d01 = make_float2(s.colc[0][lane], s.colc[0][lane + 32]);
            const float2 d23 = make_float2(s.colc[0][lane + 64], s.colc[0][lane + 96]);
            const float2 cd01 = make_float2(s.colc[3][lane], s.colc[3][lane + 32]);
            const float2 cd23 = make_float2(s.colc[3][lane + 64], s.colc[3][lane + 96]);
            float *dst = p.dense_out ? p.dense_out + (int64_t(c.req) * H + c.head) * FK * FV : nullptr;
#pragma unroll 1
            for (int g = 0; g < 4; ++g) {
                float2 X[4][2];
                tm_ld16(c.tm + 16 * g, X);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int k = warp * 16 + 4 * g + i;
                    const float2 kk = hi2(s.rowa[k]);
                    X[i][0] = pfma2(kk, d01, pmul2(X[i][0], cd01));
                    X[i][1] = pfma2(kk, d23, pmul2(X[i][1], cd23));
                    row_partial(rowpart, k, lane, X[i]);
                    if (dst) {
                        float *row = dst + k * FV + lane;
                        row[0] = X[i][0].x;
                        row[32] = X[i][0].y;
                        row[64] = X[i][1].x;
                        row[96] = X[i][1].y;
                    }
                }
                tm_st16(c.tm + 16 * g, X);
            }
        }
        tm_wait_st();
        __syncwarp();  // a warp's row partials are written and finished by that warp alone
        // Lanes j and j+16 finish row 16*warp + j: S_l = ((A_l + A_{l+8}) + A_{l+16}) + A_{l+24},
        // total = S_0 + S_1 + ... + S_7 in order.
        const int j = lane & 15, half = lane >> 4;
        const int k = warp * 16 + j;
        const float *row = rowpart + k * kRowPartStride + 4 * half;
        const float4 a0 = *reinterpret_cast<const float4 *>(row);
        const float4 a1 = *reinterpret_cast<const float4 *>(row + 8);
        const float4 a2 = *reinterpret_cast<const float4 *>(row + 16);
        const float4 a3 = *reinterpret_cast<const float4 *>(row + 24);
        const float s0 = __fadd_rn(__fadd_rn(__fadd_rn(a0.x, a1.x), a2.x), a3.x);
        const float s1 = __fadd_rn(__fadd_rn(__fadd_rn(a0.y, a1.y), a2.y), a3.y);
        const float s2 = __fadd_rn(__fadd_rn(__fadd_rn(a0.z, a1.z), a2.z), a3.z);
        const float s3 = __fadd_rn(__fadd_rn(__fadd_rn(a0.w, a1.w), a2.w), a3.w);
        float total = half ? 0.f : __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(0.f, s0), s1), s2), s3);
        const float prefix = __shfl_sync(0xffffffffu, total, j);
        if (half) {
            total = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(prefix, s0), s1), s2), s3);
            const float w = st.imp[k];
            const float mean = __fmul_rn(total, 1.f / float(FV));  // FV is a power of two: the same rounding as total / FV
            const float rr = fp16_scale(__fsqrt_rn(__fdiv_rn(fmaxf(mean, 1e-20f), w)));
            const float rc = __frcp_rn(rr);
            const float w2 = __fmul_rn(w, w);
            s.rowa[k] = make_float4(rr, rr, rc, rc);
            s.rowb[k] = make_float4(-rr, -rr, w2, w2);
            huge = !(total <= 7.922816251426434e28f);  // 2^96, or NaN
        }
        // The warp's new row constants are read by the warp alone (its P3 - P5 rows).
        __syncwarp();
        warp_slow = __any_sync(0xffffffffu, huge);
    }
    fast_quantize(s, c, float((1 << (width - 1)) - 1), warp_slow, consumed);
    if (width == 4) fast_store<4>(s, c);
    else if (width == 6) fast_store<6>(s, c);
    else fast_store<8>(s, c);
}

// Persistent kernel, one CTA per SM: CTA b owns the contiguous item range
// [b * items / grid, (b + 1) * items / grid) (item = request * H + head) and
// its item groups take the range's items one at a time from a shared
// counter, so a group that runs ahead takes more items and the groups of an SM
// finish together.  Each group keeps the next item's data in flight while it
// computes the current one, and the slot of the item after that in a small
// ring, so each item starts with its page, scales and inputs on chip.  The
// readout and decode keep two stage buffers and issue the next item's copies
// first; the step, writeback and encode keep one (the other's space holds their
// row partials and code bytes) and refill it once the item's staged data is
// consumed, before the quantizer's column passes.
template <int MODE, int G>
__global__ void __launch_bounds__(G * kThreads, 1) fast_kernel(TileParams p, int items) {
    constexpr int kGroups = G;
    // The pivot-head or 2-bit-head kernel launched after this one may start its
    // CTAs on SMs this grid leaves (it shares no data with it).
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
    extern __shared__ __align__(16) unsigned char smem_raw[];
    FastCta<kGroups> &cta = *reinterpret_cast<FastCta<kGroups> *>(smem_raw);
    const int group = threadIdx.x / kThreads;
    FastSmem &s = cta.grp[group];
    const sq_plan &P = p.plan;
    const int H = P.heads;
    Ctx c;
    c.tid = threadIdx.x % kThreads;
    c.warp = c.tid >> 5;
    c.lane = c.tid & 31;
    c.bar = 1 + group;
    const int lo = int(int64_t(blockIdx.x) * items / gridDim.x);
    const int hi = int(int64_t(blockIdx.x + 1) * items / gridDim.x);
    const int hshift = (H & (H - 1)) == 0 ? __ffs(H) - 1 : -1;
    auto request_of = [&](int it) { return hshift >= 0 ? it >> hshift : it / H; };
    // The group's first two items are lo + group and lo + kGroups + group; the
    // rest come from the counter.  Their slots are requested before the head
    // table is read so the two global round trips overlap.
    if (c.tid == 0) {
        const int i0 = lo + group, i1 = lo + kGroups + group;
        s.item_ring[0] = i0;
        s.item_ring[1] = i1;
        if (i0 < hi) cp_async8(&s.slot_ring[0], p.slots + request_of(i0));
        if (i1 < hi) cp_async8(&s.slot_ring[1], p.slots + request_of(i1));
    }
    cp_async_commit();
    for (int h = c.tid; h < H; h += kThreads) {
        HeadInfo hi;
        hi.width = P.bits[h * FK];
        hi.off_head = P.offsets[h * FK];
        hi.rows = P.rows[h * FK];
        hi.columns = P.columns[h];
        const bool gates = MODE != kWriteback && p.step.a_log;
        hi.a_log = gates ? p.step.a_log[h] : 0.f;
        hi.dt_bias = gates ? p.step.dt_bias[h] : 0.f;
        s.head[h] = hi;
    }
    if (threadIdx.x == 0) cta.next = lo + 2 * kGroups;
    if (tm_mode<MODE>() && threadIdx.x < 32) tm_alloc(&cta.grp[0].tmem_slot, 512);
    cp_async_wait<0>();
    if (tm_mode<MODE>()) tm_fence_before();
    __syncthreads();
    if (tm_mode<MODE>()) {
        tm_fence_after();
        c.tm = cta.grp[0].tmem_slot + (uint32_t(32 * (c.warp & 3)) << 16) + uint32_t(128 * group + 64 * (c.warp >> 2));
    }
    int item = s.item_ring[0];
    long long slot = s.slot_ring[0];
    if (item < hi) {
        const int req = request_of(item);
        const WorkItem first = describe(p, s, req, item - req * H, slot);
        if (first.fast && first.active) prefetch<MODE>(p, s, s.st0, first, c.tid);
    }
    cp_async_commit();
    cp_async_wait<0>();
    group_sync(c.bar);
    // Invariant at the top of round r: the current item's data is in
    // s.stage(buf), and the next item and its slot are in item_ring and
    // slot_ring[(r + 1) % 3].  Round r fills entry (r + 2) % 3, last read
    // before the barrier that ended round r - 1.
    constexpr bool kOneStage = tm_mode<MODE>();
    int buf = 0, ring = 0;  // ring = r % 3
    while (item < hi) {
        const int ring1 = ring == 2 ? 0 : ring + 1, ring2 = ring1 == 2 ? 0 : ring1 + 1;
        const int next_item = s.item_ring[ring1];
        auto issue_next = [&]() {
            if (next_item < hi) {
                const int nreq = request_of(next_item);
                const WorkItem nxt = describe(p, s, nreq, next_item - nreq * H, s.slot_ring[ring1]);
                if (nxt.fast && nxt.active) prefetch<MODE>(p, s, s.stage(kOneStage ? 0 : buf ^ 1), nxt, c.tid);
                if (c.tid == 0) {
                    const int after = atomicAdd(&cta.next, 1);
                    s.item_ring[ring2] = after;
                    if (after < hi) cp_async8(&s.slot_ring[ring2], p.slots + request_of(after));
                }
            } else if (c.tid == 0) {
                s.item_ring[ring2] = hi;
            }
            cp_async_commit();
        };
        if (!kOneStage) issue_next();
        const int req = request_of(item);
        const WorkItem cur = describe(p, s, req, item - req * H, slot);
        c.req = cur.req;
        c.head = cur.head;
        c.slot = cur.slot;
        if (MODE == kReadout && c.head == 0 && c.tid == 0) p.stable_slots[c.req] = c.slot;
        const bool body = cur.fast && cur.active;
        if (kOneStage && !body) issue_next();
        if (cur.fast) {
            if (cur.active) {
                c.page = p.pages + c.slot * P.page_bytes;
                c.off_head = s.head[c.head].off_head;
                if constexpr (kOneStage) fast_body<MODE>(p, s, s.st0, c, cur.width, issue_next);
                else fast_body<MODE>(p, s, s.stage(buf), c, cur.width, [] {});
            } else {
                if (cur.slot > 0 && c.tid == 0) flag(p.status, SQ_STATUS_SLOT_RANGE);
                if ((MODE == kStep || MODE == kReadout) && c.tid < FV)
                    store_from_float(p.step.out, p.step.io_dtype, (int64_t(c.req) * H + c.head) * FV + c.tid, 0.f);
                if ((MODE == kStep || MODE == kDecode) && p.dense_out) {
                    float *dst = p.dense_out + (int64_t(c.req) * H + c.head) * FK * FV;
                    for (int e = c.tid; e < FK * FV; e += kThreads) dst[e] = 0.f;
                }
            }
        }
        cp_async_wait<0>();  // the next item's data and the slot after it
        group_sync(c.bar);   // ... visible to the group; the stage buffer just read is free
        slot = s.slot_ring[ring1];
        item = next_item;
        if (!kOneStage) buf ^= 1;
        ring = ring1;
    }
    if (tm_mode<MODE>()) {
        tm_fence_before();
        __syncthreads();
        tm_fence_after();
        if (threadIdx.x < 32) tm_dealloc(cta.grp[0].tmem_slot, 512);
    }
}

// ---------------------------------------------------------------------------
// fp16 pivot heads: one CTA per (request, pivot head).  Step and readout alike
// read the head's values, form the column partials of k^T Y and q^T Y, the
// gates and the readout (the operations of fast_body with unit row and column
// scales), and write the updated values back as fp16 -- the reference's
// readout stores pivot rows itself, so the writeback has nothing to do for
// them.  Encode and decode convert between fp32 and fp16.
// ---------------------------------------------------------------------------
struct PivotSmem {
    float4 rowa[FK];  // {1, 1, k, k}: raw k, then the normalised k
    float4 rowb[FK];  // {q, q, -, -} raw q
    float red[2][8][FV];
    float colc[4][FV];  // [0] delta, [3] decay (c = 1)
    float misc[64];
};

template <int MODE>
__global__ void __launch_bounds__(kThreads) pivot_kernel(TileParams p, PivotHeads ph) {
    // Launched as a programmatic dependent of the readout's (step's) persistent
    // kernel, whose heads it does not touch, its CTAs fill SMs as that kernel's
    // CTAs leave; each still waits for that kernel's completion before it
    // exits, so work after it in the stream sees both (a no-op otherwise).
    struct AfterPrimary {
        __device__ ~AfterPrimary() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
    } after_primary;
    __shared__ PivotSmem s;
    const sq_plan &P = p.plan;
    const int H = P.heads;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int req = blockIdx.x / ph.count, head = ph.ids[blockIdx.x % ph.count];
    const int64_t item = int64_t(req) * H + head;
    const long long slot = p.slots[req];
    if (!(slot > 0 && slot < p.num_slots)) {
        if (slot > 0 && tid == 0) flag(p.status, SQ_STATUS_SLOT_RANGE);
        if ((MODE == kStep || MODE == kReadout) && tid < FV) store_from_float(p.step.out, p.step.io_dtype, item * FV + tid, 0.f);
        if ((MODE == kStep || MODE == kDecode) && p.dense_out)
            for (int e = tid; e < FK * FV; e += kThreads) p.dense_out[item * FK * FV + e] = 0.f;
        return;
    }
    uint8_t *values = p.pages + slot * P.page_bytes + P.offsets[head * FK];
    if (MODE == kEncode) {
        pivot_encode(p.dense_in + item * FK * FV, values, warp, lane);
        return;
    }
    if (MODE == kDecode) {
        pivot_decode(values, p.dense_out + item * FK * FV, warp, lane);
        return;
    }
    // The warp's rows first: their loads overlap the input loads and norms below.
    uint2 raw[16];
    {
        const uint8_t *src = pivot_lane(values, warp, lane);
#pragma unroll
        for (int r = 0; r < 16; ++r) raw[r] = *reinterpret_cast<const uint2 *>(src + r * 32);
    }
    const sq_step_args &a = p.step;
    float qraw = 0.f, kraw = 0.f, vin = 0.f, braw = 0.f, graw = 0.f;
    if (tid < FK) {
        const int qh = head / (H / a.qk_heads);
        qraw = load_as_float(a.q, a.io_dtype, int64_t(req) * a.q_stride + int64_t(qh) * FK + tid);
        kraw = load_as_float(a.k, a.io_dtype, int64_t(req) * a.k_stride + int64_t(qh) * FK + tid);
        vin = load_as_float(a.v, a.io_dtype, int64_t(req) * a.v_stride + int64_t(head) * FV + tid);
        braw = load_as_float(a.beta, a.gate_dtype, item);
        graw = load_as_float(a.g, a.gate_dtype, item);
        s.rowa[tid] = make_float4(1.f, 1.f, kraw, kraw);
        s.rowb[tid] = make_float4(qraw, qraw, 0.f, 0.f);
        float3 part = make_float3(__fmul_rn(qraw, qraw), __fmul_rn(kraw, kraw), __fmul_rn(qraw, kraw));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            part.x += __shfl_xor_sync(0xffffffffu, part.x, o);
            part.y += __shfl_xor_sync(0xffffffffu, part.y, o);
            part.z += __shfl_xor_sync(0xffffffffu, part.z, o);
        }
        if (lane == 0) *reinterpret_cast<float4 *>(&s.misc[4 * warp]) = make_float4(part.x, part.y, part.z, 0.f);
    }
    __syncthreads();
    pivot_rows_held(s, raw, warp, lane);
    __syncthreads();
    if (tid < FV) {
        const float beta = a.a_log ? 1.f / (1.f + expf(-braw)) : braw;
        float g = graw;
        if (a.a_log) {
            const float u = g + a.dt_bias[head];
            g = -expf(a.a_log[head]) * (u > 20.f ? u : logf(1.f + expf(fminf(u, 20.f))));
        }
        const float decay = expf(g);
        float qq = 0.f, kk = 0.f, dot = 0.f;
#pragma unroll
        for (int w = 0; w < FK / 32; ++w) {
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
        const float kS = __fmul_rn(__fmul_rn(ks, kn), decay);
        const float qS = __fmul_rn(__fmul_rn(qs, qscale), decay);
        const float delta = __fmul_rn(beta, __fsub_rn(vin, kS));
        const float kx = __fmul_rn(kraw, kn);
        s.colc[0][tid] = delta;
        s.colc[3][tid] = decay;
        s.rowa[tid].z = kx;
        s.rowa[tid].w = kx;
        store_from_float(a.out, a.io_dtype, item * FV + tid, __fmaf_rn(qk, delta, qS));
    }
    __syncthreads();
    pivot_update_held(s, raw, values, warp, lane, MODE == kStep && p.dense_out ? p.dense_out + item * FK * FV : nullptr);
}

// Resident CTAs per SM for each mode, and SMs, per device (set up on the first
// launch on a device).
constexpr int kMaxDevices = 64;
std::atomic<int> g_ready[kFit + 1][2][kMaxDevices];  // kernel attributes set, by Mode and group-count variant
std::atomic<int> g_sms[kMaxDevices];

// SMs the kernels of `stream` run on: its green context's SM partition (a
// writeback stream with an SM budget), else the whole device.  A persistent
// grid sized for more SMs than its stream owns would leave CTAs waiting for
// others to exit, each with a fixed share of the items.
int stream_sms(cudaStream_t stream, int device_sms) {
    static PFN_cuStreamGetGreenCtx_v12040 get_ctx = nullptr;
    static PFN_cuGreenCtxGetDevResource_v12040 get_res = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuStreamGetGreenCtx", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_ctx = reinterpret_cast<PFN_cuStreamGetGreenCtx_v12040>(f);
        f = nullptr;
        if (cudaGetDriverEntryPoint("cuGreenCtxGetDevResource", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_res = reinterpret_cast<PFN_cuGreenCtxGetDevResource_v12040>(f);
        (void)cudaGetLastError();
    });
    if (!stream || !get_ctx || !get_res) return device_sms;
    CUgreenCtx green = nullptr;
    if (get_ctx(reinterpret_cast<CUstream>(stream), &green) != CUDA_SUCCESS || !green) return device_sms;
    CUdevResource res;
    if (get_res(green, &res, CU_DEV_RESOURCE_TYPE_SM) != CUDA_SUCCESS) return device_sms;
    return std::max(1, std::min(device_sms, int(res.sm.smCount)));
}

// The writeback's per-SM item counts at which four 64-register item groups
// end sooner than three 80-register ones.  With n items on an SM, three groups
// end on a round one or two items wide when n = 3m + 1 or 3m + 2; four groups
// run that tail wider (n = 4, 7, 8, 10, 11; measured at 7, 8 and 11).  Beyond
// a dozen items the four-group build's extra instructions (rematerialised
// addresses, a few spills) cost more than the tail it saves (measured at 14).
// Per-rank item counts this small come from sharding value heads over many
// GPUs (1,024 items on 148 SMs at 8 GPUs of config 1: 7 on most SMs).
inline bool writeback_four_groups(int items, int grid) {
    const int n = (items + grid - 1) / grid;
    return n == 4 || n == 7 || n == 8 || n == 10 || n == 11;
}

template <int MODE, int G>
cudaError_t launch_fast_groups(const TileParams &p, int items, int device, int sms, cudaStream_t stream) {
    constexpr int smem = int(sizeof(FastCta<G>));
    std::atomic<int> *ready = device < kMaxDevices ? &g_ready[MODE][G == groups_of<MODE>() ? 0 : 1][device] : nullptr;
    if (!ready || !ready->load(std::memory_order_relaxed)) {
        const cudaError_t err = cudaFuncSetAttribute(fast_kernel<MODE, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (err != cudaSuccess) return err;
        if (ready) ready->store(1, std::memory_order_relaxed);
    }
    // One CTA per SM of the stream (its green context's SMs, if it has one),
    // each with a contiguous share of the items.
    const int grid = std::max(1, std::min(items, sms));
    fast_kernel<MODE, G><<<grid, G * kThreads, smem, stream>>>(p, items);
    return cudaGetLastError();
}

template <int MODE>
cudaError_t launch_fast_mode(const TileParams &p, int items, cudaStream_t stream) {
    int device = 0;
    cudaError_t err = cudaGetDevice(&device);
    if (err != cudaSuccess) return err;
    int sms = device < kMaxDevices ? g_sms[device].load(std::memory_order_relaxed) : 0;
    if (sms == 0) {
        if ((err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device)) != cudaSuccess) return err;
        if (device < kMaxDevices) g_sms[device].store(sms, std::memory_order_relaxed);
    }
    sms = stream_sms(stream, sms);
    if constexpr (MODE == kWriteback) {
        if (writeback_four_groups(items, std::max(1, std::min(items, sms))))
            return launch_fast_groups<MODE, 4>(p, items, device, sms, stream);
    }
    return launch_fast_groups<MODE, groups_of<MODE>()>(p, items, device, sms, stream);
}

}  // namespace

bool fast_eligible(const sq_plan &plan, const void *pages) {
    return plan.architecture == SQ_GDN && plan.storage == 0 && plan.keys == FK && plan.values == FV &&
           plan.heads <= kMaxHeads &&
           plan.page_bytes % 16 == 0 &&
           (reinterpret_cast<uintptr_t>(pages) & 15u) == 0;
}

namespace {
bool aligned16(const void *ptr, int64_t stride_bytes) {
    return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0 && stride_bytes % 16 == 0;
}
}  // namespace

cudaError_t launch_fast(int mode, const TileParams &params, int batch, cudaStream_t stream) {
    const int items = batch * params.plan.heads;
    if (items <= 0) return cudaSuccess;
    TileParams p = params;
    if (mode == kWriteback) {
        p.stage_inputs = aligned16(p.scratch, p.scratch_stride * 4);
        p.stage_gates = 0;
    } else {
        const sq_step_args &a = p.step;
        const int64_t esize = a.io_dtype == SQ_F32 ? 4 : 2;
        p.stage_inputs = aligned16(a.q, a.q_stride * esize) && aligned16(a.k, a.k_stride * esize) &&
                         aligned16(a.v, a.v_stride * esize);
        p.stage_gates = a.gate_dtype == SQ_F32 && (reinterpret_cast<uintptr_t>(a.g) & 3u) == 0 &&
                        (reinterpret_cast<uintptr_t>(a.beta) & 3u) == 0;
    }
    cudaError_t err;
    switch (mode) {
        case kStep: err = launch_fast_mode<kStep>(p, items, stream); break;
        case kReadout: err = launch_fast_mode<kReadout>(p, items, stream); break;
        case kWriteback: err = launch_fast_mode<kWriteback>(p, items, stream); break;
        case kEncode: err = launch_fast_mode<kEncode>(p, items, stream); break;
        case kDecode: err = launch_fast_mode<kDecode>(p, items, stream); break;
        default: return cudaErrorNotSupported;
    }
    if (err != cudaSuccess) return err;
    TwoHeads th;
    const bool twos = two_heads(p.plan, &th) && th.count > 0;
    if (twos && (err = launch_two(mode, p, th, batch, stream)) != cudaSuccess) return err;
    if (mode == kWriteback) return cudaSuccess;
    PivotHeads ph;
    if (!pivot_heads(p.plan, &ph) || ph.count == 0) return cudaSuccess;
    const int grid = batch * ph.count;
    if ((mode == kReadout || mode == kStep) && !twos) {
        // Directly after the persistent kernel: a programmatic dependent launch.
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(unsigned(grid));
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = 0;
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        return mode == kReadout ? cudaLaunchKernelEx(&cfg, pivot_kernel<kReadout>, p, ph)
                                : cudaLaunchKernelEx(&cfg, pivot_kernel<kStep>, p, ph);
    }
    switch (mode) {
        case kStep: pivot_kernel<kStep><<<grid, kThreads, 0, stream>>>(p, ph); break;
        case kReadout: pivot_kernel<kReadout><<<grid, kThreads, 0, stream>>>(p, ph); break;
        case kEncode: pivot_kernel<kEncode><<<grid, kThreads, 0, stream>>>(p, ph); break;
        default: pivot_kernel<kDecode><<<grid, kThreads, 0, stream>>>(p, ph); break;
    }
    return cudaGetLastError();
}

bool pivot_heads(const sq_plan &plan, PivotHeads *out) {
    out->count = 0;
    if (plan.architecture != SQ_GDN || plan.keys != FK || plan.values != FV || plan.storage != 0 || !plan.bits_host)
        return false;
    for (int h = 0; h < plan.heads; ++h) {
        if (plan.bits_host[h * plan.keys] != 16) continue;
        if (out->count == kMaxPivotHeads) return false;
        out->ids[out->count++] = h;
    }
    return true;
}


namespace {
// Lanes are processed in pairs through divide2 (the packed form the decode
// kernels use); an odd tail element goes through the scalar div_fp16.
__global__ void division_selftest_kernel(const float *a, const uint16_t *b, float *out, int64_t n) {
    const int64_t pairs = n / 2;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < pairs; i += int64_t(gridDim.x) * blockDim.x) {
        const float2 d = make_float2(__half2float(__ushort_as_half(b[2 * i])), __half2float(__ushort_as_half(b[2 * i + 1])));
        const float2 rd = make_float2(__frcp_rn(d.x), __frcp_rn(d.y));
        const float2 q = divide2<false>(make_float2(a[2 * i], a[2 * i + 1]), d, rd, make_float2(-d.x, -d.y));
        out[2 * i] = q.x;
        out[2 * i + 1] = q.y;
    }
    if (n & 1 && blockIdx.x == 0 && threadIdx.x == 0) {
        const float d = __half2float(__ushort_as_half(b[n - 1]));
        out[n - 1] = div_fp16(a[n - 1], d, __frcp_rn(d));
    }
}
}  // namespace

cudaError_t launch_division_selftest(const float *a, const uint16_t *b, float *out, int64_t n, cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    const int blocks = int(n < 4096 * 256 ? (n + 255) / 256 : 4096);
    division_selftest_kernel<<<blocks, 256, 0, stream>>>(a, b, out, n);
    return cudaGetLastError();
}

}  // namespace sq
