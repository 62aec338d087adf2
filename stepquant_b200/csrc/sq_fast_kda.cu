// Register-resident decode kernels for KDA heads with K = V = 128 (the served
// shape of Kimi-Linear-style layers): per key row a code width of 2, 4, 6 or
// 8 bits (3 and 5 with the width extension) or an fp16 pivot row, per-channel
// decay, value tile 4.
//
// One 256-thread CTA per (request, value head), three per SM (six for the
// readout, which holds no state in tensor memory and launches without the
// code plane).  The head's code bytes are staged by cp.async from a 16-byte
// cover.  Warp w owns rows 16w..16w+15 and thread (w, l) the columns l, l+32,
// l+64, l+96 of each (both torch sum orders thread-local): P1 decodes each
// value straight from the staged bytes, dequantizes and decays it (x = level *
// r_old * 2^(8-b) * decay_k * c, pivot rows value * decay_k) and forms the
// column partials of k^T S and q^T S, P2 applies the rank-1 update and the row
// |x| sums, P3-P5 evaluate fit_state for KDA rows (limit = qmax 2^(8-b),
// y = x / r / c / 2^(8-b), pivot rows excluded from c and the least squares),
// and a cooperative pass packs the codes into the staged region, which is
// written back whole.  P3-P5 divide by rn = r 2^(8-b) instead of r and then
// by c: RN(x / rn) = RN(x / r) 2^(b-8) exactly (a power-of-two scaling of a
// normal float; a quotient small enough to be subnormal has level 0 either
// way), so y needs no separate scaling.  Divisions by fp16 scales (and their
// power-of-two multiples) and by qmax (1..127: at most 7 significant bits) use
// the corrected reciprocal of the GDN kernels, exact for such divisors.
#include "sq_fast.cuh"

namespace sq {
namespace {

constexpr int DK = 128;
constexpr int DV = 128;
constexpr int DTILES = DV / 4;                 // value tiles of 4
constexpr int kCodeStage = kKdaCodeCap + 32;    // + 16-byte cover at both ends
constexpr int kRowPart = 36;                    // floats per row in the row-partial exchange

struct KdaSmem {
    unsigned char codes[kCodeStage];
    int bits[DK];
    int offs[DK];
    int rows[DK];
    float imp[DK];
    float red[2][8][DV];
    float4 rowa[DK];  // P1: {fa, fa, k, k}          P3-P5: {rn, rn, 1/rn, 1/rn}   rn = r 2^(8-b)
    float4 rowb[DK];  // P1: {q, q, isint, -}        P3-P5: {-rn, -rn, w2, w2}
    float4 rowd[DK];  // P3-P5: {-, 1/qmax (0: pivot row), qmax, isint}
    float rscale[DK]; // P3-: r (the fp16 row scale the page stores; 1 for pivot rows)
    int4 rowdec[DK];  // P1 (step, writeback): {staged byte of the row's chunk in tile 0, bits per code
                      //   (16: fp16 row), code mask (0: fp16 row), level bias -(2^23 + offset) as float bits}
    float colc[4][DV];
    float misc[64];
    int flags;
    int qmax_max;        // largest qmax of the head's integer rows
    int rho_bits;        // max over columns of RN(M' / c1) (float bits; P5 clamps)
    uint32_t tmem_slot;  // tensor-memory base of the CTA's state columns
    // Last, so that the readout, which goes without it, launches without it.
    union alignas(16) {
        float rowpart[DK * kRowPart];    // P2 row partials
        unsigned char code[DK * DV];     // P5 -> pack: the code of value v of row k at k * DV + v
    } u;
};

// Step and writeback keep each thread's 64 state values in its tensor-memory
// lane between phases (128 columns per CTA; warps w and w + 4 share a lane
// quarter with 64 columns each) and bring 16 at a time into registers.
constexpr uint32_t kTmCols = 128;

__device__ __forceinline__ int qmax_i(int b) { return (1 << ((b > 8 ? 8 : b) - 1)) - 1; }

// Row decode of the step and writeback (P1 straight from the staged bytes).
// Value v of row k (width b) sits in value tile v / 4 at bit (v % 4) b of the
// tile's chunk, which starts at the row's offset plus (v / 4) * stride; a
// thread's four values share v % 4 = lane % 4 and lie in tiles lane / 4 + 8 j.
// For an integer row the two bytes from the code's first one hold it
// (a 6-bit code can straddle a byte boundary; the second byte may be past the
// row's chunk, inside the staged region); a pivot row's value is its fp16.
struct KdaRowDecode {
    int at;       // staged byte of the lane's code in tile lane / 4 (add 8 j stride for the others)
    uint32_t sh;  // its bit shift inside those two bytes
    uint32_t mask;  // (1 << b) - 1; 0 for a pivot row
    float bias;   // -(2^23 + offset)
};

__device__ __forceinline__ float kda_staged_value(const unsigned char *codes, const KdaRowDecode &d, int j_off) {
    if (d.mask == 0u) return __half2float(*reinterpret_cast<const __half *>(codes + d.at + j_off));
    const uint32_t u = uint32_t(codes[d.at + j_off]) | (uint32_t(codes[d.at + j_off + 1]) << 8);
    return __fadd_rn(__uint_as_float(0x4B000000u | ((u >> d.sh) & d.mask)), d.bias);
}

// P1 of the readout, which keeps no state: lane l covers the four consecutive
// columns 4l .. 4l + 3 (value tile l), decoded straight from the staged code
// bytes instead of through the fp16 plane.  Each element is formed with the
// same operations as in P1 of the step (the level is exact either way), and
// each column's partial is the same ordered sum over the warp's 16 rows, so
// the results are identical.
__device__ __forceinline__ void kda_readout_rows(KdaSmem &s, int lead, int off0, int stride, int warp, int lane) {
    const float4 c = *reinterpret_cast<const float4 *>(&s.colc[3][4 * lane]);
    const float2 c01 = make_float2(c.x, c.y), c23 = make_float2(c.z, c.w), one = make_float2(1.f, 1.f);
    const int base = lead - off0 + lane * stride;
    const uint32_t *words = reinterpret_cast<const uint32_t *>(s.codes);
    float2 kx01 = make_float2(0.f, 0.f), kx23 = kx01, qx01 = kx01, qx23 = kx01;
#pragma unroll 2
    for (int r = 0; r < 16; ++r) {
        const int k = warp * 16 + r;
        const float4 a = s.rowa[k];
        const float4 d = s.rowb[k];  // {q, level bias, code mask (0: fp16 row), byte offset of the row}
        const int at = base + __float_as_int(d.w);
        // The chunk's first 4 (fp16: 8) bytes from aligned words; the staged
        // region has 16 spare bytes past its end, so the reads stay inside it.
        const uint32_t *w = words + (at >> 2);
        const uint32_t sh = uint32_t(at & 3) * 8u;
        const uint32_t w0 = __funnelshift_r(w[0], w[1], sh);
        const uint32_t mask = __float_as_uint(d.z);
        float2 v01, v23;
        if (mask == 0u) {  // fp16 row (the width is the row's: the branch is warp-uniform)
            const uint32_t w1 = __funnelshift_r(w[1], w[2], sh);
            v01 = __half22float2(*reinterpret_cast<const __half2 *>(&w0));
            v23 = __half22float2(*reinterpret_cast<const __half2 *>(&w1));
        } else {  // 2^23 + code - (2^23 + offset) = level, exactly
            const int b = __popc(mask);
            const float2 bias = make_float2(d.y, d.y);
            v01 = __fadd2_rn(make_float2(__uint_as_float(0x4B000000u | (w0 & mask)),
                                         __uint_as_float(0x4B000000u | ((w0 >> b) & mask))), bias);
            v23 = __fadd2_rn(make_float2(__uint_as_float(0x4B000000u | ((w0 >> (2 * b)) & mask)),
                                         __uint_as_float(0x4B000000u | ((w0 >> (3 * b)) & mask))), bias);
        }
        const bool integer = mask != 0u;
        const float2 m01 = integer ? c01 : one, m23 = integer ? c23 : one;
        const float2 x01 = pmul2(pmul2(v01, lo2(a)), m01);
        const float2 x23 = pmul2(pmul2(v23, lo2(a)), m23);
        const float2 q = make_float2(d.x, d.x);
        kx01 = pfma2(hi2(a), x01, kx01);
        kx23 = pfma2(hi2(a), x23, kx23);
        qx01 = pfma2(q, x01, qx01);
        qx23 = pfma2(q, x23, qx23);
    }
    *reinterpret_cast<float4 *>(&s.red[0][warp][4 * lane]) = make_float4(kx01.x, kx01.y, kx23.x, kx23.y);
    *reinterpret_cast<float4 *>(&s.red[1][warp][4 * lane]) = make_float4(qx01.x, qx01.y, qx23.x, qx23.y);
}

// P3 partial: per column, the maximum over the warp's integer rows of
// |x / r| / limit = |x / rn| / qmax -> s.red[0].  EXACT divides (corrected
// reciprocals, IEEE on the SLOW path); otherwise |x| * RN(1/rn) * RN(1/qmax),
// whose relative distance from the exact value is below 6 * 2^-24 (six float
// steps), bounds it.  (A maximum in the subnormal range gives c0 = fp16's
// smallest scale whatever its value.)
template <bool SLOW, bool EXACT>
__device__ __forceinline__ void kda_column_max(KdaSmem &s, int warp, int lane, uint32_t tm) {
    float m0 = 0.f, m1 = 0.f, m2 = 0.f, m3 = 0.f;
#pragma unroll 1
    for (int g = 0; g < 4; ++g) {
        float2 X[4][2];
        tm_ld16(tm + 16 * g, X);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int k = warp * 16 + 4 * g + i;
            const float4 a = s.rowa[k], b = s.rowb[k], d = s.rowd[k];
            const float keep = d.w;
            float2 t01, t23;
            if (EXACT) {
                const float2 qm = make_float2(d.z, d.z), rq = make_float2(d.y, d.y), nq = make_float2(-d.z, -d.z);
                const float2 s01 = divide2<SLOW>(X[i][0], lo2(a), hi2(a), lo2(b));
                const float2 s23 = divide2<SLOW>(X[i][1], lo2(a), hi2(a), lo2(b));
                t01 = divide2<SLOW>(make_float2(fabsf(s01.x), fabsf(s01.y)), qm, rq, nq);
                t23 = divide2<SLOW>(make_float2(fabsf(s23.x), fabsf(s23.y)), qm, rq, nq);
            } else {
                const float2 rl = make_float2(d.y, d.y);
                t01 = pmul2(pmul2(make_float2(fabsf(X[i][0].x), fabsf(X[i][0].y)), hi2(a)), rl);
                t23 = pmul2(pmul2(make_float2(fabsf(X[i][1].x), fabsf(X[i][1].y)), hi2(a)), rl);
            }
            // (pivot rows: 1/qmax is 0 in the row table, so the products and
            // the corrected-reciprocal quotients are 0; IEEE quotients are masked)
            m0 = fmaxf(m0, SLOW ? t01.x * keep : t01.x);
            m1 = fmaxf(m1, SLOW ? t01.y * keep : t01.y);
            m2 = fmaxf(m2, SLOW ? t23.x * keep : t23.x);
            m3 = fmaxf(m3, SLOW ? t23.y * keep : t23.y);
        }
    }
    s.red[0][warp][lane] = m0;
    s.red[0][warp][lane + 32] = m1;
    s.red[0][warp][lane + 64] = m2;
    s.red[0][warp][lane + 96] = m3;
}

// P4 body: first levels and the weighted least-squares sums; the thread's
// values go from x to x / rn in tensor memory (rn = 1 for pivot rows).
template <bool SLOW, bool CLAMP>
__device__ __forceinline__ void kda_first_levels(const KdaSmem &s, int warp, int lane, uint32_t tm, float2 (&num)[2],
                                                 float2 (&den)[2]) {
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
            const int k = warp * 16 + 4 * g + i;
            const float4 a = s.rowa[k], b = s.rowb[k], d = s.rowd[k];
            const float2 rn = lo2(a), w2 = hi2(b);
            const float q = d.z;
            const bool integer = d.w != 0.f;
            const float2 nrk = pmul2(rn, nround);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const float2 x = X[i][h];
                const float2 sn = divide2<SLOW>(x, rn, hi2(a), lo2(b));
                float2 y = divide2<SLOW>(sn, h ? c23 : c01, h ? r23 : r01, h ? n23 : n01);
                // Pivot rows (weight 0 in the sums) are always clamped: their
                // unbounded levels could overflow v * v and turn 0 * inf into NaN.
                if (CLAMP || !integer) y = clamp2(y, q);
                const float2 v = pfma2(rn, __fadd2_rn(y, round), nrk);
                num[h] = __fadd2_rn(num[h], product_term(pmul2(w2, v), x));
                den[h] = __fadd2_rn(den[h], product_term(w2, pmul2(v, v)));
                X[i][h] = sn;  // (pivot rows: rn = 1, so sn is x exactly)
            }
        }
        tm_st16(tm + 16 * g, X);
    }
    tm_wait_st();
}

// P5 body: final levels of integer rows -> their code bytes in the byte plane
// (code = level + offset: the low byte of RN(y + 1.5 2^23) plus the offset);
// pivot rows -> their fp16 values straight into the staged region (the
// lane's value of tile lane / 4 + 8 j at `pivot_at` + 8 j stride + the row's offset).
// CLAMP: rows whose qmax times `rho` (the largest RN(M'/c1) of the tile's
// columns) can exceed qmax + 1/2 clamp their levels; the others cannot reach
// the clamp (|y| <= qmax M / c1 for a row with that qmax).
template <bool SLOW, bool CLAMP>
__device__ __forceinline__ void kda_final_levels(KdaSmem &s, int warp, int lane, uint32_t tm, int pivot_at, int j8,
                                                 float rho) {
    const float2 c01 = make_float2(s.colc[1][lane], s.colc[1][lane + 32]);
    const float2 c23 = make_float2(s.colc[1][lane + 64], s.colc[1][lane + 96]);
    const float2 r01 = make_float2(s.colc[2][lane], s.colc[2][lane + 32]);
    const float2 r23 = make_float2(s.colc[2][lane + 64], s.colc[2][lane + 96]);
    const float2 n01 = make_float2(-c01.x, -c01.y), n23 = make_float2(-c23.x, -c23.y);
    const float2 round = make_float2(kRound, kRound);
#pragma unroll 1
    for (int g = 0; g < 4; ++g) {
        float2 X[4][2];
        tm_ld16(tm + 16 * g, X);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int k = warp * 16 + 4 * g + i;
            const float4 d = s.rowd[k];
            if (d.w != 0.f) {
                unsigned char *code = s.u.code + k * DV + lane;
                const uint32_t off = uint32_t(d.z);
                const bool clamp = CLAMP && (SLOW || !(__fmul_rn(rho, d.z) <= d.z + 0.49f));  // warp-uniform (row k)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    float2 y = divide2<SLOW>(X[i][h], h ? c23 : c01, h ? r23 : r01, h ? n23 : n01);
                    if (clamp) y = clamp2(y, d.z);
                    const float2 t = __fadd2_rn(y, round);  // low byte: the level (two's complement)
                    code[64 * h] = static_cast<unsigned char>(__float_as_uint(t.x) + off);
                    code[64 * h + 32] = static_cast<unsigned char>(__float_as_uint(t.y) + off);
                }
            } else {
                unsigned char *dst = s.codes + pivot_at + s.offs[k];
                reinterpret_cast<__half *>(dst)[0] = __float2half_rn(X[i][0].x);
                reinterpret_cast<__half *>(dst + j8)[0] = __float2half_rn(X[i][0].y);
                reinterpret_cast<__half *>(dst + 2 * j8)[0] = __float2half_rn(X[i][1].x);
                reinterpret_cast<__half *>(dst + 3 * j8)[0] = __float2half_rn(X[i][1].y);
            }
        }
    }
}

// P3-P5 on the thread's values in tensor memory.  c0 = fp16(M), M the
// column's maximum of |x/r|/limit over integer rows: the products bound M
// within six float steps; when fp16 rounds the whole interval of seven steps
// either side to one value, that is c0, otherwise the tile redoes the maxima
// with exact divisions.  Clamps are skipped when they cannot act: with c0 a
// normal, unclamped fp16 value every |x/r/c0| / 2^(8-b) < qmax_b (1 + 2^-10)
// < qmax_b + 1/2; for c1, when RN(M'/c1) * qmax_max <= qmax_max + 0.49 with M'
// the bound of M and qmax_max the head's largest qmax.  The SLOW path (huge
// or NaN rows) divides in IEEE arithmetic and always clamps.
template <bool SLOW>
__device__ __forceinline__ void kda_quantize(KdaSmem &s, int warp, int lane, int tid, uint32_t tm, int pivot_at, int j8) {
    kda_column_max<SLOW, SLOW>(s, warp, lane, tm);
    __syncthreads();
    int settled = 1;
    float mx = 0.f;  // the exact maximum, or an upper bound of it
    if (tid < DV) {
        float m = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) m = fmaxf(m, s.red[0][w][tid]);
        if (SLOW) {
            mx = m;
        } else {
            const uint32_t bits = __float_as_uint(m);
            const float lo = bits > 7u ? __uint_as_float(bits - 7u) : 0.f;
            mx = __uint_as_float(bits + 7u);
            settled = fp16_scale(lo) == fp16_scale(mx);
        }
    }
    if (!SLOW && !__syncthreads_and(settled)) {
        kda_column_max<false, true>(s, warp, lane, tm);
        __syncthreads();
        if (tid < DV) {
            mx = 0.f;
#pragma unroll
            for (int w = 0; w < 8; ++w) mx = fmaxf(mx, s.red[0][w][tid]);
        }
    }
    int safe = 1;
    if (tid == 0) s.rho_bits = 0;
    if (tid < DV) {
        const float c0 = fp16_scale(mx);
        s.colc[1][tid] = c0;
        s.colc[2][tid] = __frcp_rn(c0);
        safe = (c0 >= 6.103515625e-05f) && (mx <= 65504.f);
    }
    const bool no_clamp = __syncthreads_and(safe);
    // P4: first levels and the weighted least-squares sums.
    {
        float2 num[2], den[2];
        if (!SLOW && no_clamp) kda_first_levels<SLOW, false>(s, warp, lane, tm, num, den);
        else kda_first_levels<SLOW, true>(s, warp, lane, tm, num, den);
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
    safe = 1;
    if (tid < DV) {
        float num = 0.f, den = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) {
            num = __fadd_rn(num, s.red[0][w][tid]);
            den = __fadd_rn(den, s.red[1][w][tid]);
        }
        const float c1 = den > 0.f ? fp16_scale(__fdiv_rn(num, fmaxf(den, 1e-30f))) : s.colc[1][tid];
        s.colc[1][tid] = c1;
        s.colc[2][tid] = __frcp_rn(c1);
        const float qm = float(s.qmax_max);
        const float rho = c1 >= 6.103515625e-05f ? __fdiv_rn(mx, c1) : __int_as_float(0x7f800000);
        atomicMax(&s.rho_bits, __float_as_int(rho));  // non-negative floats order as their bits (NaN above all)
        safe = (c1 >= 6.103515625e-05f) && (__fmul_rn(rho, qm) <= qm + 0.49f);
    }
    const bool no_clamp5 = __syncthreads_and(safe);
    // P5: final levels (integer rows) or the fp16 values (pivot rows) -> plane.
    const float rho = __int_as_float(s.rho_bits);
    if (!SLOW && no_clamp5) kda_final_levels<SLOW, false>(s, warp, lane, tm, pivot_at, j8, rho);
    else kda_final_levels<SLOW, true>(s, warp, lane, tm, pivot_at, j8, rho);
    __syncthreads();
}

template <int MODE>
__global__ void __launch_bounds__(kThreads, MODE == kReadout ? 6 : 3) kda_kernel(TileParams p) {
    constexpr bool kTm = MODE == kStep || MODE == kWriteback;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    KdaSmem &s = *reinterpret_cast<KdaSmem *>(smem_raw);
    const sq_plan &P = p.plan;
    const int H = P.heads;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int req = blockIdx.x / H, head = blockIdx.x % H;
    const int64_t slot = p.slots[req];
    if (MODE == kReadout && head == 0 && tid == 0) p.stable_slots[req] = slot;
    if (!fast_head_dev(P, head)) return;  // the tile kernel handles this head
    if (!(slot > 0 && slot < p.num_slots)) {
        if (slot > 0 && tid == 0) flag(p.status, SQ_STATUS_SLOT_RANGE);
        if (MODE != kWriteback && tid < DV)
            store_from_float(p.step.out, p.step.io_dtype, (int64_t(req) * H + head) * DV + tid, 0.f);
        if (MODE == kStep && p.dense_out) {
            float *dst = p.dense_out + (int64_t(req) * H + head) * DK * DV;
            for (int e = tid; e < DK * DV; e += kThreads) dst[e] = 0.f;
        }
        return;
    }
    uint8_t *page = p.pages + slot * P.page_bytes;
    const int stride = P.offsets[H * DK + head];
    const int off0 = P.offsets[head * DK];
    const int coff = P.columns[head];

    // ---- stage the code region (16-byte cover), per-row tables, inputs ------
    const uintptr_t a0 = reinterpret_cast<uintptr_t>(page + off0);
    const uintptr_t base = a0 & ~uintptr_t(15);
    const int lead = int(a0 - base);
    {
        const int span = lead + stride * DTILES;
        for (int j = tid; 16 * j < span; j += kThreads)
            cp_async16(s.codes + 16 * j, reinterpret_cast<const void *>(base + 16 * uintptr_t(j)));
    }
    float qx = 0.f, kx = 0.f, vin = 0.f, ga = 0.f, rold = 1.f, cold = 0.f, decay = 1.f, delta = 0.f;
    int bk = 16;
    if (tid < DK) {
        bk = P.bits[head * DK + tid];
        s.bits[tid] = bk;
        s.offs[tid] = P.offsets[head * DK + tid];
        const int ro = P.rows[head * DK + tid];
        s.rows[tid] = ro;
        s.imp[tid] = P.impact[head * DK + tid];
        if (ro >= 0) rold = half_at(page, ro);
        cold = half_at(page, coff + 2 * tid);
        if (MODE == kWriteback) {
            const float *sc = p.scratch + int64_t(req) * p.scratch_stride + int64_t(head) * (DV + 2 * DK);
            delta = sc[tid];
            kx = sc[DV + tid];
            decay = sc[DV + DK + tid];
        } else {
            const sq_step_args &a = p.step;
            const int qh = head / (H / a.qk_heads);
            qx = load_as_float(a.q, a.io_dtype, int64_t(req) * a.q_stride + int64_t(qh) * DK + tid);
            kx = load_as_float(a.k, a.io_dtype, int64_t(req) * a.k_stride + int64_t(qh) * DK + tid);
            vin = load_as_float(a.v, a.io_dtype, int64_t(req) * a.v_stride + int64_t(head) * DV + tid);
            ga = load_as_float(a.g, a.gate_dtype, (int64_t(req) * H + head) * DK + tid);
        }
    }
    float beta = 0.f, qk = 0.f;
    if (MODE != kWriteback) {
        const sq_step_args &a = p.step;
        float3 part = make_float3(__fmul_rn(qx, qx), __fmul_rn(kx, kx), __fmul_rn(qx, kx));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            part.x += __shfl_xor_sync(0xffffffffu, part.x, o);
            part.y += __shfl_xor_sync(0xffffffffu, part.y, o);
            part.z += __shfl_xor_sync(0xffffffffu, part.z, o);
        }
        if (lane == 0) {
            s.misc[4 * warp] = part.x;
            s.misc[4 * warp + 1] = part.y;
            s.misc[4 * warp + 2] = part.z;
        }
        if (tid < DK) {  // DK == DV: the threads that finish the columns
            const float braw = load_as_float(a.beta, a.gate_dtype, int64_t(req) * H + head);
            beta = a.a_log ? 1.f / (1.f + expf(-braw)) : braw;
            float g = ga;
            if (a.a_log) {
                const float u = g + a.dt_bias[head * DK + tid];
                g = -expf(a.a_log[head]) * (u > 20.f ? u : logf(1.f + expf(fminf(u, 20.f))));
            }
            decay = expf(g);
        }
    }
    if (kTm && warp == 0) tm_alloc(&s.tmem_slot, kTmCols);
    asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;\n" ::: "memory");
    if (kTm) tm_fence_before();
    __syncthreads();
    uint32_t tm = 0;  // the thread's 64 columns: value (row 4g+i, half h, lane e) at 16g + 4i + 2h + e
    if (kTm) {
        tm_fence_after();
        tm = s.tmem_slot + (uint32_t(32 * (warp & 3)) << 16) + uint32_t(64 * (warp >> 2));
    }
    if (MODE != kWriteback && tid < DK) {
        const sq_step_args &a = p.step;
        float qq = 0.f, kk = 0.f, dot = 0.f;
#pragma unroll
        for (int w = 0; w < kThreads / 32; ++w) {
            const float4 m = reinterpret_cast<const float4 *>(s.misc)[w];
            qq += m.x;
            kk += m.y;
            dot += m.z;
        }
        const float qn = a.normalize ? __frsqrt_rn(qq + 1e-6f) : 1.f;
        const float kn = a.normalize ? __frsqrt_rn(kk + 1e-6f) : 1.f;
        qx = __fmul_rn(__fmul_rn(qx, qn), a.scale);
        kx = __fmul_rn(kx, kn);
        qk = __fmul_rn(__fmul_rn(__fmul_rn(dot, qn), kn), a.scale);
    }
    if (tid < DK) {
        const bool integer = bk != 16;
        const float norm = integer ? float(1 << (8 - (bk > 8 ? 8 : bk))) : 1.f;
        const float fa = integer ? __fmul_rn(__fmul_rn(rold, norm), decay) : decay;
        s.rowa[tid] = make_float4(fa, fa, kx, kx);
        if (MODE == kReadout)  // the readout's row decode table (kda_readout_rows)
            s.rowb[tid] = make_float4(qx, integer ? -(8388608.f + float(qmax_i(bk))) : 0.f,
                                      __uint_as_float(integer ? (1u << bk) - 1u : 0u), __int_as_float(s.offs[tid]));
        else  // {q, -, integer row, width}
            s.rowb[tid] = make_float4(qx, qx, integer ? 1.f : 0.f, __int_as_float(bk));
        if (MODE != kReadout)
            s.rowdec[tid] = make_int4(lead - off0 + s.offs[tid], integer ? bk : 16, integer ? int((1u << bk) - 1u) : 0,
                                      __float_as_int(-(8388608.f + float(qmax_i(bk)))));
        s.colc[3][tid] = cold;
        if (MODE == kWriteback) s.colc[0][tid] = delta;
    }
    __syncthreads();

    // ---- P1: dequantize and decay; column partials of k^T S and q^T S -------
    {
        const float2 c01 = make_float2(s.colc[3][lane], s.colc[3][lane + 32]);
        const float2 c23 = make_float2(s.colc[3][lane + 64], s.colc[3][lane + 96]);
        const float2 one = make_float2(1.f, 1.f);
        float2 kx01 = make_float2(0.f, 0.f), kx23 = kx01, qx01 = kx01, qx23 = kx01;
        if (MODE == kReadout) kda_readout_rows(s, lead, off0, stride, warp, lane);
        const int e = lane & 3, tile_at = (lane >> 2) * stride, j8 = 8 * stride;
#pragma unroll 1
        for (int g = 0; g < (MODE == kReadout ? 0 : 4); ++g) {
            float2 X[4][2];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int k = warp * 16 + 4 * g + i;
                const float4 a = s.rowa[k], b = s.rowb[k];
                KdaRowDecode d;
                {
                    const int4 rd = s.rowdec[k];
                    const int pos = e * rd.y;  // fp16 rows: 16 e, i.e. byte 2 e, shift 0
                    d.at = rd.x + tile_at + (pos >> 3);
                    d.sh = uint32_t(pos & 7);
                    d.mask = uint32_t(rd.z);
                    d.bias = __int_as_float(rd.w);
                }
                const float2 v01 = make_float2(kda_staged_value(s.codes, d, 0), kda_staged_value(s.codes, d, j8));
                const float2 v23 = make_float2(kda_staged_value(s.codes, d, 2 * j8), kda_staged_value(s.codes, d, 3 * j8));
                const bool integer = d.mask != 0u;
                const float2 m01 = integer ? c01 : one, m23 = integer ? c23 : one;
                const float2 x01 = pmul2(pmul2(v01, lo2(a)), m01);
                const float2 x23 = pmul2(pmul2(v23, lo2(a)), m23);
                X[i][0] = x01;
                X[i][1] = x23;
                kx01 = pfma2(hi2(a), x01, kx01);
                kx23 = pfma2(hi2(a), x23, kx23);
                qx01 = pfma2(lo2(b), x01, qx01);
                qx23 = pfma2(lo2(b), x23, qx23);
            }
            if (kTm) tm_st16(tm + 16 * g, X);
        }
        if (MODE == kStep) {
            s.red[0][warp][lane] = kx01.x;
            s.red[0][warp][lane + 32] = kx01.y;
            s.red[0][warp][lane + 64] = kx23.x;
            s.red[0][warp][lane + 96] = kx23.y;
            s.red[1][warp][lane] = qx01.x;
            s.red[1][warp][lane + 32] = qx01.y;
            s.red[1][warp][lane + 64] = qx23.x;
            s.red[1][warp][lane + 96] = qx23.y;
        }
        if (MODE != kWriteback) {
            __syncthreads();
            if (tid < DV) {
                float ks = 0.f, qs = 0.f;
#pragma unroll
                for (int w = 0; w < 8; ++w) {
                    ks = __fadd_rn(ks, s.red[0][w][tid]);
                    qs = __fadd_rn(qs, s.red[1][w][tid]);
                }
                const float d = __fmul_rn(beta, __fsub_rn(vin, ks));
                s.colc[0][tid] = d;
                store_from_float(p.step.out, p.step.io_dtype, (int64_t(req) * H + head) * DV + tid, __fmaf_rn(qk, d, qs));
                if (MODE == kReadout) {
                    float *sc = p.scratch + int64_t(req) * p.scratch_stride + int64_t(head) * (DV + 2 * DK);
                    sc[tid] = d;
                    sc[DV + tid] = kx;
                    sc[DV + DK + tid] = decay;
                }
            }
        }
        // The readout writes no page bytes: the writeback rewrites each head's
        // code region whole (pivot rows included, recomputed from the same inputs).
        if (MODE == kReadout) return;
        __syncthreads();  // P1 reads of the plane are done before P2 writes row partials over it
    }

    // ---- P2: rank-1 update; row sums of |x| in torch order; row constants ----
    {
        const float2 d01 = make_float2(s.colc[0][lane], s.colc[0][lane + 32]);
        const float2 d23 = make_float2(s.colc[0][lane + 64], s.colc[0][lane + 96]);
        float *rowpart = s.u.rowpart;
        float *dst = MODE == kStep && p.dense_out ? p.dense_out + (int64_t(req) * H + head) * DK * DV : nullptr;
#pragma unroll 1
        for (int g = 0; g < 4; ++g) {
            float2 X[4][2];
            tm_ld16(tm + 16 * g, X);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int k = warp * 16 + 4 * g + i;
                const float2 kk = hi2(s.rowa[k]);
                X[i][0] = pfma2(kk, d01, X[i][0]);
                X[i][1] = pfma2(kk, d23, X[i][1]);
                rowpart[k * kRowPart + lane] = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(0.f, fabsf(X[i][0].x)),
                                                                             fabsf(X[i][0].y)), fabsf(X[i][1].x)),
                                                         fabsf(X[i][1].y));
                if (dst) {
                    float *row = dst + k * DV + lane;
                    row[0] = X[i][0].x;
                    row[32] = X[i][0].y;
                    row[64] = X[i][1].x;
                    row[96] = X[i][1].y;
                }
            }
            tm_st16(tm + 16 * g, X);
        }
        tm_wait_st();
        if (tid == 0) {
            s.flags = 0;
            s.qmax_max = 0;
        }
        __syncthreads();
        const int j = lane & 15, half = lane >> 4;
        const int k = warp * 16 + j;
        const float *row = rowpart + k * kRowPart + 4 * half;
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
            const int b = s.bits[k];
            const bool integer = b != 16;
            const float w = s.imp[k];
            const float mean = __fdiv_rn(total, float(DV));
            float rr = fp16_scale(__fsqrt_rn(__fdiv_rn(fmaxf(mean, 1e-20f), w)));
            if (!integer) rr = 1.f;
            const float w2 = integer ? __fmul_rn(w, w) : 0.f;
            const int bb = b > 8 ? 8 : b;
            const float norm = float(1 << (8 - bb)), inv = __uint_as_float(uint32_t(127 - 8 + bb) << 23);
            // rn = r 2^(8-b) and RN(1/rn) = RN(1/r) 2^(b-8): exact power-of-two scalings
            const float rn = __fmul_rn(rr, norm), rcn = __fmul_rn(__frcp_rn(rr), inv);
            const float qm = float(qmax_i(b));
            s.rowa[k] = make_float4(rn, rn, rcn, rcn);
            s.rowb[k] = make_float4(-rn, -rn, w2, w2);
            s.rowd[k] = make_float4(0.f, integer ? __frcp_rn(qm) : 0.f, qm, integer ? 1.f : 0.f);
            s.rscale[k] = rr;
            if (integer) atomicMax(&s.qmax_max, qmax_i(b));
            if (integer && !(total <= 7.922816251426434e28f)) atomicOr(&s.flags, 1);  // 2^96, or NaN
        }
    }
    __syncthreads();
    {
        const int pivot_at = lead - off0 + (lane >> 2) * stride + 2 * (lane & 3);
        if (s.flags) kda_quantize<true>(s, warp, lane, tid, tm, pivot_at, 8 * stride);
        else kda_quantize<false>(s, warp, lane, tid, tm, pivot_at, 8 * stride);
    }

    // ---- pack the integer rows' codes into the staged region ----------------
    // Chunk (k, t): the four code bytes of values 4t..4t+3 (one word of the
    // byte plane), the code of value 4t + i moved to bit i b; b / 2 bytes.
    for (int idx = tid; idx < DK * DTILES; idx += kThreads) {
        const int k = idx >> 5, t = idx & 31;
        const int b = s.bits[k];
        if (b == 16) continue;  // pivot values were stored in P5
        unsigned char *dst = s.codes + lead + (s.offs[k] - off0) + t * stride;
        const uint32_t w = *reinterpret_cast<const uint32_t *>(&s.u.code[k * DV + 4 * t]);
        const uint32_t m = (1u << b) - 1u;
        const uint32_t packed = (w & m) | ((w >> (8 - b)) & (m << b)) | ((w >> (16 - 2 * b)) & (m << (2 * b))) |
                                ((w >> (24 - 3 * b)) & (m << (3 * b)));
        dst[0] = uint8_t(packed);  // ceil(4 b / 8) bytes (3/5-bit rows of the extension end in zero bits)
        if (b >= 3) dst[1] = uint8_t(packed >> 8);
        if (b >= 5) dst[2] = uint8_t(packed >> 16);
        if (b >= 7) dst[3] = uint8_t(packed >> 24);
    }
    __syncthreads();
    // ---- write the head's code region back: whole 16-byte pieces as vectors,
    // the ragged first and last pieces byte by byte (their other bytes belong
    // to neighbouring heads or pages).  Alignment padding inside the region
    // keeps the staged (prior) bytes.
    {
        const uintptr_t a_end = a0 + uintptr_t(stride) * DTILES;
        for (int j = tid; base + 16 * uintptr_t(j) < a_end; j += kThreads) {
            const uintptr_t g = base + 16 * uintptr_t(j);
            if (g >= a0 && g + 16 <= a_end) {
                *reinterpret_cast<uint4 *>(g) = *reinterpret_cast<const uint4 *>(s.codes + 16 * j);
            } else {
                for (int e = 0; e < 16; ++e)
                    if (g + e >= a0 && g + e < a_end) *reinterpret_cast<uint8_t *>(g + e) = s.codes[16 * j + e];
            }
        }
    }
    if (tid < DK) {
        if (s.rows[tid] >= 0) put_half(page, s.rows[tid], s.rscale[tid]);
    } else {
        put_half(page, coff + 2 * (tid - DK), s.colc[1][tid - DK]);
    }
    if (kTm) {
        tm_fence_before();
        __syncthreads();
        tm_fence_after();
        if (warp == 0) tm_dealloc(s.tmem_slot, kTmCols);
    }
}

template <int MODE>
cudaError_t launch_kda_mode(const TileParams &p, int items, cudaStream_t stream) {
    const int smem = MODE == kReadout ? int(offsetof(KdaSmem, u)) : int(sizeof(KdaSmem));
    cudaError_t err = cudaFuncSetAttribute(kda_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (err != cudaSuccess) return err;
    kda_kernel<MODE><<<items, kThreads, smem, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace

bool kda_fast_eligible(const sq_plan &plan) {
    return plan.architecture == SQ_KDA && plan.storage == 0 && plan.keys == DK && plan.values == DV;
}

cudaError_t launch_fast_kda(int mode, const TileParams &p, int batch, cudaStream_t stream) {
    const int items = batch * p.plan.heads;
    if (items <= 0) return cudaSuccess;
    switch (mode) {
        case kStep: return launch_kda_mode<kStep>(p, items, stream);
        case kReadout: return launch_kda_mode<kReadout>(p, items, stream);
        case kWriteback: return launch_kda_mode<kWriteback>(p, items, stream);
        default: return cudaErrorNotSupported;
    }
}

}  // namespace sq
