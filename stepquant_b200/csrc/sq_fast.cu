// Register-resident decode kernels for GDN heads with K = V = 128 and a code
// width of 4, 6 or 8 bits (the served shape of Qwen-Next-style layers).
//
// One 256-thread CTA per (request, value head); two CTAs per SM.  Warp w owns
// key rows 16w..16w+15 and lane l owns value columns l, l+32, l+64, l+96, so
// each thread keeps 64 state elements in registers for the whole step.  That
// mapping makes both ordered sums of fit_state local:
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
#include "sq_tile.cuh"

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

struct FastSmem {
    unsigned char stage[kTiles * (FK * 16 + kStagePad)];  // old packed codes, padded per tile
    unsigned char plane[kPlaneBytes];                     // row partials, then new code bytes
    float red[2][8][FV];                                  // per-warp column partials
    float4 rowc[FK];                                      // per-row constants
    float colc[4][FV];                                    // per-column constants
    __half rold[FK];
    __half cold[FV];
    float qv[FK];
    float kv[FK];
    float misc[64];
    int flags;
};

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\n" ::);
    asm volatile("cp.async.wait_group 0;\n" ::);
}

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

// Signed level (code - offset) of value-lane u of row k in value tile t, read
// from the staged page; exact small integers built with the 2^23 trick.
template <int BITS>
__device__ __forceinline__ float staged_level(const unsigned char *stage, int t, int k, int u) {
    const unsigned char *chunk = stage + t * (W<BITS>::tile_bytes + kStagePad) + k * W<BITS>::chunk;
    if (BITS == 8) {
        const uint32_t c = chunk[u];
        return __fsub_rn(__uint_as_float(0x4B000000u | c), 8388608.f + float(W<BITS>::off));
    } else if (BITS == 4) {
        const uint32_t byte = chunk[u >> 1];
        const int s = 4 * (u & 1);
        const uint32_t m = byte & (0xFu << s);
        const float scale = s ? 0.0625f : 1.f;
        return __fmaf_rn(__uint_as_float(0x4B000000u | m), scale, -(8388608.f * scale + float(W<BITS>::off)));
    } else {
        const int bit = 6 * u;
        const int p = bit >> 3, s = bit & 7;
        const uint32_t w = uint32_t(chunk[p]) | (uint32_t(chunk[p + 1]) << 8);
        const uint32_t m = w & (0x3Fu << s);
        const float scale = __uint_as_float(uint32_t(127 - s) << 23);  // 2^-s
        return __fmaf_rn(__uint_as_float(0x4B000000u | m), scale, -(8388608.f * scale + float(W<BITS>::off)));
    }
}

// Pack 16 code bytes (one per value lane) of chunk (t, k) from the plane into
// the page's 2*BITS-byte little-endian chunk.
template <int BITS>
__device__ __forceinline__ void store_chunk(uint8_t *dst, const unsigned char *plane_chunk) {
    const uint4 w = *reinterpret_cast<const uint4 *>(plane_chunk);
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
    int req, head, warp, lane, tid;
    int64_t slot;
    uint8_t *page;
    int off_head;
};

// P3-P5: column max -> c0; first levels and the weighted least-squares sums
// -> c1; final levels -> code plane -> packed page chunks; r and c stores.
template <int BITS, int MODE, bool SLOW>
__device__ __forceinline__ void fast_quantize(const TileParams &p, FastSmem &s, const Ctx &c, float (&X)[16][4]) {
    const sq_plan &P = p.plan;
    const int warp = c.warp, lane = c.lane, tid = c.tid;
    constexpr float qmax = float(W<BITS>::off);
    // P3: c0 = fp16(max_k |x / r| / qmax) (uniform width: one division per column).
    {
        float m[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int r = 0; r < 16; ++r) {
            const float4 rc = s.rowc[warp * 16 + r];
#pragma unroll
            for (int i = 0; i < 4; ++i) m[i] = fmaxf(m[i], fabsf(divide<SLOW>(X[r][i], rc.x, rc.y)));
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) s.red[0][warp][lane + 32 * i] = m[i];
    }
    __syncthreads();
    int safe = 1;
    if (tid < FV) {
        float mx = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) mx = fmaxf(mx, s.red[0][w][tid]);
        const float ratio = __fdiv_rn(mx, qmax);
        const float c0 = fp16_scale(ratio);
        s.colc[1][tid] = c0;
        s.colc[2][tid] = __frcp_rn(c0);
        // With c0 a normal, unclamped fp16 value every |x/r/c0| < qmax + 1/2: no clamp needed.
        safe = (c0 >= 6.103515625e-05f) && (ratio <= 65504.f);
    }
    const bool no_clamp = __syncthreads_and(safe);
    // P4: first levels, weighted least-squares numerator / denominator (16-row blocks).
    {
        float c0[4], rc0[4], num[4] = {0.f, 0.f, 0.f, 0.f}, den[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            c0[i] = s.colc[1][lane + 32 * i];
            rc0[i] = s.colc[2][lane + 32 * i];
        }
#pragma unroll
        for (int r = 0; r < 16; ++r) {
            const float4 rc = s.rowc[warp * 16 + r];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float x = X[r][i];
                const float sn = divide<SLOW>(x, rc.x, rc.y);
                float z = rintf(divide<SLOW>(sn, c0[i], rc0[i]));
                if (!no_clamp) z = fminf(fmaxf(z, -qmax), qmax);
                const float v = __fmul_rn(rc.x, z);
                num[i] = __fadd_rn(num[i], __fmul_rn(__fmul_rn(rc.z, v), x));
                den[i] = __fadd_rn(den[i], __fmul_rn(rc.z, __fmul_rn(v, v)));
                X[r][i] = sn;
            }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            s.red[0][warp][lane + 32 * i] = num[i];
            s.red[1][warp][lane + 32 * i] = den[i];
        }
    }
    __syncthreads();
    if (tid < FV) {
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
    // P5: final levels -> one code byte per value in the plane.
    {
        float c1[4], rc1[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            c1[i] = s.colc[1][lane + 32 * i];
            rc1[i] = s.colc[2][lane + 32 * i];
        }
        const int t0 = lane >> 4, u = lane & 15;
#pragma unroll
        for (int r = 0; r < 16; ++r) {
            const int k = warp * 16 + r;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float z = fminf(fmaxf(rintf(divide<SLOW>(X[r][i], c1[i], rc1[i])), -qmax), qmax);
                const uint32_t code = __float_as_uint(__fadd_rn(z, 8388608.f + qmax));
                s.plane[(t0 + 2 * i) * (FK * 16 + kStagePad) + k * 16 + u] = static_cast<unsigned char>(code);
            }
        }
    }
    __syncthreads();
    // Pack the plane into the page and store the scales.
    {
        uint8_t *dst = c.page + c.off_head;
        const int stride = W<BITS>::tile_bytes;
        for (int ch = tid; ch < kTiles * FK; ch += kThreads) {
            const int t = ch / FK, k = ch % FK;
            store_chunk<BITS>(dst + t * stride + k * W<BITS>::chunk, s.plane + t * (FK * 16 + kStagePad) + k * 16);
        }
        if (tid < FK) {
            reinterpret_cast<__half *>(c.page + P.rows[c.head * FK])[tid] = __float2half_rn(s.rowc[tid].x);
        } else {
            reinterpret_cast<__half *>(c.page + P.columns[c.head])[tid - FK] = __float2half_rn(s.colc[1][tid - FK]);
        }
    }
}

// ---------------------------------------------------------------------------
// The per-head body.  MODE: kStep (fused), kReadout, kWriteback.
// ---------------------------------------------------------------------------
template <int BITS, int MODE>
__device__ void fast_body(const TileParams &p, FastSmem &s, const Ctx &c) {
    const sq_plan &P = p.plan;
    const int H = P.heads;
    const int warp = c.warp, lane = c.lane, tid = c.tid;
    uint8_t *page = c.page;

    // ---- stage the head's codes, r and c (cp.async, 16-byte pieces) --------
    {
        const uint8_t *src = page + c.off_head;
        constexpr int pieces = W<BITS>::head_bytes / 16;
        constexpr int per_tile = W<BITS>::tile_bytes / 16;
        for (int j = tid; j < pieces; j += kThreads) {
            const int t = j / per_tile, within = j % per_tile;
            cp_async16(s.stage + t * (W<BITS>::tile_bytes + kStagePad) + within * 16, src + j * 16);
        }
        const int rowoff = P.rows[c.head * FK];
        const int coloff = P.columns[c.head];
        if (tid < 16) cp_async16(reinterpret_cast<unsigned char *>(s.rold) + tid * 16, page + rowoff + tid * 16);
        else if (tid < 32) cp_async16(reinterpret_cast<unsigned char *>(s.cold) + (tid - 16) * 16, page + coloff + (tid - 16) * 16);
    }

    // ---- per-request inputs ------------------------------------------------
    float beta = 0.f, qk = 0.f, decay = 1.f;
    if (MODE == kWriteback) {
        const float *sc = p.scratch + int64_t(c.req) * p.scratch_stride + int64_t(c.head) * (FV + 2 * FK);
        if (tid < FK) {
            s.colc[0][tid] = sc[tid];          // delta
            s.kv[tid] = sc[FV + tid];          // normalised k
        }
        decay = sc[FV + FK];
    } else {
        const sq_step_args &a = p.step;
        const int qh = c.head / (H / a.qk_heads);
        float qq = 0.f, kk = 0.f, qkp = 0.f;
        if (tid < FK) {
            const float qx = load_as_float(a.q, a.io_dtype, int64_t(c.req) * a.q_stride + int64_t(qh) * FK + tid);
            const float kx = load_as_float(a.k, a.io_dtype, int64_t(c.req) * a.k_stride + int64_t(qh) * FK + tid);
            s.qv[tid] = qx;
            s.kv[tid] = kx;
            qq = __fmul_rn(qx, qx);
            kk = __fmul_rn(kx, kx);
            s.colc[3][tid] = load_as_float(a.v, a.io_dtype, int64_t(c.req) * a.v_stride + int64_t(c.head) * FV + tid);
        }
        float qn = 1.f, kn = 1.f;
        if (a.normalize) {
            qn = __frsqrt_rn(block_sum(qq, s.misc) + 1e-6f);
            kn = __frsqrt_rn(block_sum(kk, s.misc) + 1e-6f);
        }
        if (tid < FK) {
            const float qx = __fmul_rn(__fmul_rn(s.qv[tid], qn), a.scale);
            const float kx = __fmul_rn(s.kv[tid], kn);
            s.qv[tid] = qx;
            s.kv[tid] = kx;
            qkp = __fmul_rn(qx, kx);
        }
        qk = block_sum(qkp, s.misc);
        const float braw = load_as_float(a.beta, a.gate_dtype, int64_t(c.req) * H + c.head);
        beta = a.a_log ? 1.f / (1.f + expf(-braw)) : braw;
        float g = load_as_float(a.g, a.gate_dtype, int64_t(c.req) * H + c.head);
        if (a.a_log) {
            const float u = g + a.dt_bias[c.head];
            g = -expf(a.a_log[c.head]) * (u > 20.f ? u : logf(1.f + expf(fminf(u, 20.f))));
        }
        decay = expf(g);
    }
    cp_async_wait_all();
    __syncthreads();
    if (tid < FK) s.rowc[tid] = make_float4(__fmul_rn(__half2float(s.rold[tid]), decay), s.kv[tid], s.qv[tid], 0.f);
    __syncthreads();

    // ---- P1: unpack, dequantize, decay; column partials of k^T S and q^T S ---
    float X[16][4];
    float colc_old[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) colc_old[i] = __half2float(s.cold[lane + 32 * i]);
    const int t0 = lane >> 4, u = lane & 15;
    {
        float kx[4] = {0.f, 0.f, 0.f, 0.f}, qx[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int r = 0; r < 16; ++r) {
            const int k = warp * 16 + r;
            const float4 rc = s.rowc[k];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float z = staged_level<BITS>(s.stage, t0 + 2 * i, k, u);
                const float x = __fmul_rn(__fmul_rn(z, rc.x), colc_old[i]);
                X[r][i] = x;
                kx[i] = __fmaf_rn(rc.y, x, kx[i]);
                qx[i] = __fmaf_rn(rc.z, x, qx[i]);
            }
        }
        if (MODE != kWriteback) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                s.red[0][warp][lane + 32 * i] = kx[i];
                s.red[1][warp][lane + 32 * i] = qx[i];
            }
            __syncthreads();
            if (tid < FV) {
                float ks = 0.f, qs = 0.f;
#pragma unroll
                for (int w = 0; w < 8; ++w) {
                    ks = __fadd_rn(ks, s.red[0][w][tid]);
                    qs = __fadd_rn(qs, s.red[1][w][tid]);
                }
                const float delta = __fmul_rn(beta, __fsub_rn(s.colc[3][tid], ks));
                s.colc[0][tid] = delta;
                const float out = __fmaf_rn(qk, delta, qs);
                store_from_float(p.step.out, p.step.io_dtype, (int64_t(c.req) * H + c.head) * FV + tid, out);
                if (MODE == kReadout) {
                    float *sc = p.scratch + int64_t(c.req) * p.scratch_stride + int64_t(c.head) * (FV + 2 * FK);
                    sc[tid] = delta;
                    sc[FV + tid] = s.kv[tid];
                    sc[FV + FK + tid] = decay;
                }
            }
            if (MODE == kReadout) return;
            __syncthreads();
        }
    }

    // ---- P2: rank-1 update; row sums of |x| in torch order; new row scales ---
    float delta[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) delta[i] = s.colc[0][lane + 32 * i];
    float *rowpart = reinterpret_cast<float *>(s.plane);
#pragma unroll
    for (int r = 0; r < 16; ++r) {
        const int k = warp * 16 + r;
        const float kk = s.rowc[k].y;
        float a = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            X[r][i] = __fmaf_rn(kk, delta[i], X[r][i]);
            a = __fadd_rn(a, fabsf(X[r][i]));
        }
        rowpart[k * kRowPartStride + lane] = a;
    }
    if (MODE == kStep && p.dense_out) {
        float *dst = p.dense_out + (int64_t(c.req) * H + c.head) * FK * FV;
#pragma unroll
        for (int r = 0; r < 16; ++r)
#pragma unroll
            for (int i = 0; i < 4; ++i) dst[(warp * 16 + r) * FV + lane + 32 * i] = X[r][i];
    }
    if (tid == 0) s.flags = 0;
    __syncthreads();
    {
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
            const float w = P.impact[c.head * FK + k];
            const float mean = __fdiv_rn(total, float(FV));
            const float r = fp16_scale(__fsqrt_rn(__fdiv_rn(fmaxf(mean, 1e-20f), w)));
            s.rowc[k] = make_float4(r, __frcp_rn(r), __fmul_rn(w, w), 0.f);
            if (!(total <= 7.922816251426434e28f)) atomicOr(&s.flags, 1);  // 2^96, or NaN
        }
    }
    __syncthreads();
    if (s.flags) {
        // Pathological magnitudes: IEEE divisions for the whole tile.
        fast_quantize<BITS, MODE, true>(p, s, c, X);
    } else {
        fast_quantize<BITS, MODE, false>(p, s, c, X);
    }
}


template <int MODE>
__global__ void __launch_bounds__(kThreads, 2) fast_kernel(TileParams p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    FastSmem &s = *reinterpret_cast<FastSmem *>(smem_raw);
    const sq_plan &P = p.plan;
    const int H = P.heads;
    Ctx c;
    c.tid = threadIdx.x;
    c.warp = c.tid >> 5;
    c.lane = c.tid & 31;
    c.req = blockIdx.x / H;
    c.head = blockIdx.x % H;
    c.slot = p.slots[c.req];
    if (MODE == kReadout && c.head == 0 && c.tid == 0) p.stable_slots[c.req] = c.slot;
    const int width = P.bits[c.head * FK];
    if (width != 4 && width != 6 && width != 8) return;  // handled by the tile kernel
    bool active = c.slot > 0;
    if (active && c.slot >= p.num_slots) {
        if (c.tid == 0) flag(p.status, SQ_STATUS_SLOT_RANGE);
        active = false;
    }
    if (!active) {
        if (MODE != kWriteback && c.tid < FV)
            store_from_float(p.step.out, p.step.io_dtype, (int64_t(c.req) * H + c.head) * FV + c.tid, 0.f);
        if (MODE == kStep && p.dense_out) {
            float *dst = p.dense_out + (int64_t(c.req) * H + c.head) * FK * FV;
            for (int e = c.tid; e < FK * FV; e += kThreads) dst[e] = 0.f;
        }
        return;
    }
    c.page = p.pages + c.slot * P.page_bytes;
    c.off_head = P.offsets[c.head * FK];
    if (width == 4) fast_body<4, MODE>(p, s, c);
    else if (width == 6) fast_body<6, MODE>(p, s, c);
    else fast_body<8, MODE>(p, s, c);
}

template <int MODE>
cudaError_t launch_fast_mode(const TileParams &p, int items, cudaStream_t stream) {
    const int smem = int(sizeof(FastSmem));
    cudaError_t err = cudaFuncSetAttribute(fast_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (err != cudaSuccess) return err;
    fast_kernel<MODE><<<items, kThreads, smem, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace

bool fast_eligible(const sq_plan &plan, const void *pages) {
    return plan.architecture == SQ_GDN && plan.keys == FK && plan.values == FV && plan.page_bytes % 16 == 0 &&
           (reinterpret_cast<uintptr_t>(pages) & 15u) == 0;
}

cudaError_t launch_fast(int mode, const TileParams &p, int batch, cudaStream_t stream) {
    const int items = batch * p.plan.heads;
    if (items <= 0) return cudaSuccess;
    switch (mode) {
        case kStep: return launch_fast_mode<kStep>(p, items, stream);
        case kReadout: return launch_fast_mode<kReadout>(p, items, stream);
        case kWriteback: return launch_fast_mode<kWriteback>(p, items, stream);
        default: return cudaErrorNotSupported;
    }
}


namespace {
__global__ void division_selftest_kernel(const float *a, const uint16_t *b, float *out, int64_t n) {
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
        const float d = __half2float(__ushort_as_half(b[i]));
        out[i] = div_fp16(a[i], d, __frcp_rn(d));
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
