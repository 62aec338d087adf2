// GDN chunked prefill (WY/UT form) on tensor cores, in two kernels.
//
// Within a 64-token chunk with cumulative log decay gam_i and per-token
// normalisations nk, nq (applied in fp32 to exact bf16 products of the raw
// inputs):
//   L_ij = beta_i exp(gam_i - gam_j) nk_i nk_j (k_i . k_j)          (j < i)
//   P_ij = exp(gam_i - gam_j) nq_i scale nk_j (q_i . k_j)            (j <= i)
//   T    = (I + L)^-1       (fp32: 16x16 diagonal blocks by substitution,
//                            off-diagonal blocks T_rc = -T_rr sum_m L_rm T_mc)
//   W    = T diag(beta e^gam nk) K,   U = T diag(beta) V
//   D    = U - W S                    (the chunk's beta-scaled residuals)
//   O    = diag(e^gam nq scale) Q S + P D
//   S'   = e^gam_C S + K^T diag(e^(gam_C - gam) nk) D
// which equals the token-by-token recurrence of core.delta_step.
//
// prep_kernel (one CTA per chunk and value head, all chunks in parallel)
// computes everything that does not depend on S -- P, -W, U and the row
// factors -- into a workspace record; state_kernel (one CTA per sequence and
// value head) walks the chunks in order with the 128x128 state in fp32
// registers, prefetching the next chunk's record while it computes D, O and
// the state update.  Every product is an mma.sync m16n8k16 bf16 tile with fp32
// accumulation (operands staged in padded shared memory, read with ldmatrix).
// Padded tokens of a last partial chunk have beta = 0 and log decay 0, so they
// leave the state unchanged.
#include "sq_common.cuh"

namespace sq {
namespace {

constexpr int PC = 64;    // chunk length
constexpr int PK = 128;   // keys
constexpr int PV = 128;   // values
constexpr int kLd = 136;  // bf16 row stride of 128-wide tiles (272 B: ldmatrix rows hit distinct banks)
constexpr int kLdP = 72;  // bf16 row stride of 64-wide tiles
constexpr int kLdF = 68;  // fp32 row stride of 64x64 tiles

using bf16 = __nv_bfloat16;

// Workspace record of one (chunk, value head), byte offsets.
constexpr int kRecW = 0;                   // -W   bf16 [64][128]
constexpr int kRecU = kRecW + PC * PK * 2;  // U    bf16 [64][128]
constexpr int kRecP = kRecU + PC * PV * 2;  // P    bf16 [64][64]
constexpr int kRecRo = kRecP + PC * PC * 2; // e^gam nq scale      fp32 [64]
constexpr int kRecRd = kRecRo + PC * 4;     // e^(gam_C - gam) nk  fp32 [64]
constexpr int kRecDc = kRecRd + PC * 4;     // e^gam_C             fp32 (16 bytes)
constexpr int kRec = (kRecDc + 16 + 255) / 256 * 256;
constexpr int kOffsetsBytes(int seqs) { return (4 * (seqs + 1) + 255) / 256 * 256; }

__device__ __forceinline__ unsigned smem_addr(const void *p) { return static_cast<unsigned>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ void ldsm4(uint32_t (&r)[4], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(smem_addr(p)));
}
__device__ __forceinline__ void ldsm4t(uint32_t (&r)[4], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(smem_addr(p)));
}
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void cp16(void *smem, const void *gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_addr(smem)), "l"(gmem));
}

// Fragment loads (lane l, i = l / 8, r = l % 8).
// A tile 16x16 at (m0, k0) of a row-major [m][k] matrix.
template <int LD>
__device__ __forceinline__ void load_a(uint32_t (&a)[4], const bf16 (*m)[LD], int m0, int k0, int lane) {
    const int i = lane >> 3, r = lane & 7;
    ldsm4(a, &m[m0 + r + 8 * (i & 1)][k0 + 8 * (i >> 1)]);
}
// A tile 16x16 at (m0, k0) of A = X^T, X stored row-major [k][m].
template <int LD>
__device__ __forceinline__ void load_a_t(uint32_t (&a)[4], const bf16 (*x)[LD], int m0, int k0, int lane) {
    const int i = lane >> 3, r = lane & 7;
    ldsm4t(a, &x[k0 + r + 8 * (i >> 1)][m0 + 8 * (i & 1)]);
}
// B fragments of two n-tiles (n0, n0 + 8) at k0 from B^T stored row-major [n][k]:
// b[0], b[1] for n-tile n0 and b[2], b[3] for n0 + 8.
template <int LD>
__device__ __forceinline__ void load_b_nk(uint32_t (&b)[4], const bf16 (*m)[LD], int n0, int k0, int lane) {
    const int i = lane >> 3, r = lane & 7;
    ldsm4(b, &m[n0 + r + 8 * (i >> 1)][k0 + 8 * (i & 1)]);
}
// The same from B stored row-major [k][n].
template <int LD>
__device__ __forceinline__ void load_b_kn(uint32_t (&b)[4], const bf16 (*m)[LD], int n0, int k0, int lane) {
    const int i = lane >> 3, r = lane & 7;
    ldsm4t(b, &m[k0 + r + 8 * (i & 1)][n0 + 8 * (i >> 1)]);
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&v);
}

// Token range of sequence n, clamped to [0, tokens).
__device__ __forceinline__ int2 seq_range(const sq_prefill_args &a, int n) {
    const int b = max(0, min(a.cu_seqlens[n], a.tokens));
    return make_int2(b, max(b, min(a.cu_seqlens[n + 1], a.tokens)));
}

// offsets[n] = number of chunks of the sequences before n (offsets[seqs] = all).
__global__ void __launch_bounds__(1024) offsets_kernel(sq_prefill_args a, int32_t *offsets) {
    __shared__ int warp_total[32];
    const int per = (a.num_seqs + 1023) / 1024;
    const int first = threadIdx.x * per, last = min(a.num_seqs, first + per);
    int local = 0;
    for (int n = first; n < last; ++n) {
        const int2 r = seq_range(a, n);
        local += (r.y - r.x + PC - 1) / PC;
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int run = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, run, o);
        if (lane >= o) run += y;
    }
    if (lane == 31) warp_total[warp] = run;
    __syncthreads();
    if (warp == 0) {
        int w = warp_total[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += y;
        }
        warp_total[lane] = w;  // inclusive totals
    }
    __syncthreads();
    int before = run - local + (warp ? warp_total[warp - 1] : 0);
    for (int n = first; n < last; ++n) {
        offsets[n] = before;
        const int2 r = seq_range(a, n);
        before += (r.y - r.x + PC - 1) / PC;
    }
    if (threadIdx.x == 0) offsets[a.num_seqs] = warp_total[31];
}

// ---------------------------------------------------------------------------
// prep_kernel: one 256-thread CTA per (chunk, value head).
// ---------------------------------------------------------------------------
struct PrepSmem {
    bf16 q[PC][kLd];
    bf16 k[PC][kLd];
    bf16 v[PC][kLd];
    float l[PC][kLdF];  // L; then Tu (bf16 [64][72])
    float t[PC][kLdF];  // T
    float x[PC][kLdF];  // block products; then Tw (bf16 [64][72])
    float gam[PC];
    float beta[PC];
    float nq[PC];
    float nk[PC];
};

__global__ void __launch_bounds__(256, 2) prep_kernel(sq_prefill_args a, const int32_t *offsets,
                                                      unsigned char *records) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    PrepSmem &s = *reinterpret_cast<PrepSmem *>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g8 = lane >> 2, tig = lane & 3;
    const int H = a.heads, head = blockIdx.y, chunk = blockIdx.x;
    if (chunk >= offsets[a.num_seqs]) return;
    int lo = 0, hi = a.num_seqs - 1;  // the sequence: largest n with offsets[n] <= chunk
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (offsets[mid] <= chunk) lo = mid;
        else hi = mid - 1;
    }
    const int2 range = seq_range(a, lo);
    const int t0 = range.x + (chunk - offsets[lo]) * PC, n = min(PC, range.y - t0);
    const int qh = head / (H / a.qk_heads);
    unsigned char *rec = records + (int64_t(chunk) * H + head) * kRec;

    // ---- raw q, k, v rows of the chunk (zero rows past the end), gates
    {
        const bf16 *qg = static_cast<const bf16 *>(a.q), *kg = static_cast<const bf16 *>(a.k);
        const bf16 *vg = static_cast<const bf16 *>(a.v);
        for (int idx = tid; idx < 3 * PC * 16; idx += 256) {
            const int which = idx >> 10, row = (idx >> 4) & 63, piece = idx & 15;
            bf16 *dst = (which == 0 ? s.q[row] : which == 1 ? s.k[row] : s.v[row]) + piece * 8;
            if (row < n) {
                const int64_t t = t0 + row;
                const bf16 *src = which == 0 ? qg + t * a.q_stride + int64_t(qh) * PK
                                  : which == 1 ? kg + t * a.k_stride + int64_t(qh) * PK
                                               : vg + t * a.v_stride + int64_t(head) * PV;
                cp16(dst, src + piece * 8);
            } else {
                *reinterpret_cast<uint4 *>(dst) = make_uint4(0u, 0u, 0u, 0u);
            }
        }
        if (tid < PC) {
            const bool live = tid < n;
            const int64_t gi = (int64_t(t0) + tid) * H + head;
            s.gam[tid] = live ? a.g[gi] : 0.f;
            s.beta[tid] = live ? a.beta[gi] : 0.f;
        }
        asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;\n" ::);
        __syncthreads();
    }
    // ---- norms of the q and k rows (2 threads per row), cumulative log decay
    {
        const int row = (tid >> 1) & 63, half = tid & 1;
        const bf16 *src = tid < 128 ? s.q[row] : s.k[row];
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint4 w = *reinterpret_cast<const uint4 *>(src + half * 64 + j * 8);
            const __nv_bfloat162 *h2 = reinterpret_cast<const __nv_bfloat162 *>(&w);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 f = __bfloat1622float2(h2[e]);
                ss += f.x * f.x + f.y * f.y;
            }
        }
        ss += __shfl_xor_sync(0xffffffffu, ss, 1);
        const float nrm = a.normalize ? rsqrtf(ss + 1e-6f) : 1.f;
        if (half == 0) {
            if (tid < 128) s.nq[row] = nrm;
            else s.nk[row] = nrm;
        }
    }
    if (warp == 0) {
        const float x0 = s.gam[2 * lane], x1 = s.gam[2 * lane + 1];
        float run = x0 + x1;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float y = __shfl_up_sync(0xffffffffu, run, o);
            if (lane >= o) run += y;
        }
        const float before = run - (x0 + x1);
        __syncwarp();
        s.gam[2 * lane] = before + x0;
        s.gam[2 * lane + 1] = run;
    }
    __syncthreads();

    // ---- G = K K^T, H = Q K^T (rows 16 (w / 2), columns 32 (w % 2) .. +31) -> L, P
    {
        const int r0 = 16 * (warp >> 1), c0 = 32 * (warp & 1);
        float accG[4][4] = {}, accH[4][4] = {};
#pragma unroll
        for (int ks = 0; ks < PK / 16; ++ks) {
            uint32_t ak[4], aq[4], b0[4], b1[4];
            load_a<kLd>(ak, s.k, r0, 16 * ks, lane);
            load_a<kLd>(aq, s.q, r0, 16 * ks, lane);
            load_b_nk<kLd>(b0, s.k, c0, 16 * ks, lane);
            load_b_nk<kLd>(b1, s.k, c0 + 16, 16 * ks, lane);
            mma16816(accG[0], ak, b0[0], b0[1]);
            mma16816(accG[1], ak, b0[2], b0[3]);
            mma16816(accG[2], ak, b1[0], b1[1]);
            mma16816(accG[3], ak, b1[2], b1[3]);
            mma16816(accH[0], aq, b0[0], b0[1]);
            mma16816(accH[1], aq, b0[2], b0[3]);
            mma16816(accH[2], aq, b1[0], b1[1]);
            mma16816(accH[3], aq, b1[2], b1[3]);
        }
        bf16 *prec = reinterpret_cast<bf16 *>(rec + kRecP);
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                const int i = r0 + g8 + 8 * hh, j = c0 + 8 * nt + 2 * tig;
                float pv[2];
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int jj = j + e;
                    const float dec = jj <= i ? expf(s.gam[i] - s.gam[jj]) : 0.f;
                    s.l[i][jj] = jj < i ? s.beta[i] * dec * s.nk[i] * s.nk[jj] * accG[nt][2 * hh + e] : 0.f;
                    pv[e] = dec * s.nq[i] * a.scale * s.nk[jj] * accH[nt][2 * hh + e];
                }
                *reinterpret_cast<uint32_t *>(prec + i * PC + j) = pack_bf16(pv[0], pv[1]);
            }
        }
    }
    __syncthreads();

    // ---- T = (I + L)^-1: diagonal blocks by substitution, then block rows 1..3
    if (warp < 4) {
        if (lane < 16) {
            const int b = 16 * warp, m = lane;
            float t[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                float val = i == m ? 1.f : 0.f;
#pragma unroll
                for (int j = 0; j < i; ++j) val -= s.l[b + i][b + j] * t[j];
                t[i] = val;
                s.t[b + i][b + m] = val;
            }
        }
    } else {
        for (int e = tid - 128; e < 6 * 256; e += 128) {
            const int blk = e >> 8, i = (e >> 4) & 15, m = e & 15;
            const int r = blk < 3 ? 0 : blk < 5 ? 1 : 2;
            const int c = blk < 3 ? blk + 1 : blk < 5 ? blk - 1 : 3;
            s.t[16 * r + i][16 * c + m] = 0.f;
        }
    }
    __syncthreads();
    for (int r = 1; r < 4; ++r) {
        for (int e = tid; e < r * 256; e += 256) {
            const int c = e >> 8, i = (e >> 4) & 15, m = e & 15;
            float x = 0.f;
            for (int j = 16 * c; j < 16 * r; ++j) x += s.l[16 * r + i][j] * s.t[j][16 * c + m];
            s.x[16 * r + i][16 * c + m] = x;
        }
        __syncthreads();
        for (int e = tid; e < r * 256; e += 256) {
            const int c = e >> 8, i = (e >> 4) & 15, m = e & 15;
            float t = 0.f;
#pragma unroll
            for (int j = 0; j < 16; ++j) t -= s.t[16 * r + i][16 * r + j] * s.x[16 * r + j][16 * c + m];
            s.t[16 * r + i][16 * c + m] = t;
        }
        __syncthreads();
    }

    // ---- Tw = T diag(beta e^gam nk) (into x), Tu = T diag(beta) (into l), bf16
    bf16 (*Tw)[kLdP] = reinterpret_cast<bf16 (*)[kLdP]>(&s.x[0][0]);
    bf16 (*Tu)[kLdP] = reinterpret_cast<bf16 (*)[kLdP]>(&s.l[0][0]);
    for (int e = tid; e < PC * PC; e += 256) {
        const int i = e >> 6, j = e & 63;
        const float t = s.t[i][j];
        Tw[i][j] = __float2bfloat16_rn(t * (s.beta[j] * expf(s.gam[j]) * s.nk[j]));
        Tu[i][j] = __float2bfloat16_rn(t * s.beta[j]);
    }
    __syncthreads();

    // ---- -W = -Tw K and U = Tu V (rows 16 (w % 4), columns 64 (w / 4) .. +63)
    {
        const int r0 = 16 * (warp & 3), c0 = 64 * (warp >> 2);
        float W[8][4] = {}, U[8][4] = {};
#pragma unroll
        for (int ks = 0; ks < PC / 16; ++ks) {
            uint32_t aw[4], au[4];
            load_a<kLdP>(aw, Tw, r0, 16 * ks, lane);
            load_a<kLdP>(au, Tu, r0, 16 * ks, lane);
#pragma unroll
            for (int np = 0; np < 4; ++np) {
                uint32_t bk[4], bv[4];
                load_b_kn<kLd>(bk, s.k, c0 + 16 * np, 16 * ks, lane);
                load_b_kn<kLd>(bv, s.v, c0 + 16 * np, 16 * ks, lane);
                mma16816(W[2 * np], aw, bk[0], bk[1]);
                mma16816(W[2 * np + 1], aw, bk[2], bk[3]);
                mma16816(U[2 * np], au, bv[0], bv[1]);
                mma16816(U[2 * np + 1], au, bv[2], bv[3]);
            }
        }
        bf16 *wrec = reinterpret_cast<bf16 *>(rec + kRecW);
        bf16 *urec = reinterpret_cast<bf16 *>(rec + kRecU);
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
            const int col = c0 + 8 * nt + 2 * tig, i0 = r0 + g8, i1 = i0 + 8;
            *reinterpret_cast<uint32_t *>(wrec + i0 * PK + col) = pack_bf16(-W[nt][0], -W[nt][1]);
            *reinterpret_cast<uint32_t *>(wrec + i1 * PK + col) = pack_bf16(-W[nt][2], -W[nt][3]);
            *reinterpret_cast<uint32_t *>(urec + i0 * PV + col) = pack_bf16(U[nt][0], U[nt][1]);
            *reinterpret_cast<uint32_t *>(urec + i1 * PV + col) = pack_bf16(U[nt][2], U[nt][3]);
        }
    }
    if (tid < PC) {
        const float gC = s.gam[PC - 1];
        reinterpret_cast<float *>(rec + kRecRo)[tid] = expf(s.gam[tid]) * s.nq[tid] * a.scale;
        reinterpret_cast<float *>(rec + kRecRd)[tid] = expf(gC - s.gam[tid]) * s.nk[tid];
        if (tid == 0) reinterpret_cast<float *>(rec + kRecDc)[0] = expf(gC);
    }
}

// ---------------------------------------------------------------------------
// state_kernel: one 512-thread CTA per (sequence, value head).
// ---------------------------------------------------------------------------
struct StateStage {
    bf16 w[PC][kLd];  // -W
    bf16 q[PC][kLd];  // raw q
    bf16 k[PC][kLd];  // raw k
    bf16 p[PC][kLdP];
    bf16 u[PC][PV];
    float ro[PC];
    float rd[PC];
    float dc[4];
};

struct StateSmem {
    StateStage st[2];
    bf16 s[PK][kLd];  // the state in bf16 (operand of W S and Q S)
    bf16 d[PC][kLd];  // D
    bf16 dt[PC][kLd]; // diag(e^(gam_C - gam) nk) D
};

// cp.async copies of chunk (t0, n rows) and its record into a stage.
__device__ __forceinline__ void stage_chunk(const sq_prefill_args &a, StateStage &st, const unsigned char *rec, int t0,
                                            int n, int qh, int tid) {
    const bf16 *qg = static_cast<const bf16 *>(a.q), *kg = static_cast<const bf16 *>(a.k);
    for (int idx = tid; idx < 2 * PC * 16; idx += 512) {
        const int which = idx >> 10, row = (idx >> 4) & 63, piece = idx & 15;
        bf16 *dst = (which == 0 ? st.q[row] : st.k[row]) + piece * 8;
        if (row < n) {
            const int64_t t = t0 + row;
            cp16(dst, (which == 0 ? qg + t * a.q_stride : kg + t * a.k_stride) + int64_t(qh) * PK + piece * 8);
        } else {
            *reinterpret_cast<uint4 *>(dst) = make_uint4(0u, 0u, 0u, 0u);
        }
    }
    for (int idx = tid; idx < PC * 16; idx += 512) {
        const int row = idx >> 4, piece = idx & 15;
        cp16(st.w[row] + piece * 8, rec + kRecW + row * PK * 2 + piece * 16);
        cp16(reinterpret_cast<unsigned char *>(st.u) + idx * 16, rec + kRecU + idx * 16);
    }
    for (int idx = tid; idx < PC * 8 + 33; idx += 512) {
        if (idx < PC * 8) {
            const int row = idx >> 3, piece = idx & 7;
            cp16(st.p[row] + piece * 8, rec + kRecP + row * PC * 2 + piece * 16);
        } else {
            const int j = idx - PC * 8;  // ro (16 pieces), rd (16), dc (1)
            cp16(reinterpret_cast<unsigned char *>(j < 16 ? st.ro : j < 32 ? st.rd : st.dc) + (j & 15) * 16,
                 rec + kRecRo + j * 16);
        }
    }
}

__global__ void __launch_bounds__(512, 1) state_kernel(sq_prefill_args a, const int32_t *offsets,
                                                       const unsigned char *records) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    StateSmem &s = *reinterpret_cast<StateSmem *>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g8 = lane >> 2, tig = lane & 3;
    const int H = a.heads;
    const int seq = blockIdx.x / H, head = blockIdx.x % H;
    const int qh = head / (H / a.qk_heads);
    const int2 range = seq_range(a, seq);
    const int chunks = (range.y - range.x + PC - 1) / PC;
    const unsigned char *rec0 = records + (int64_t(offsets[seq]) * H + head) * kRec;
    bf16 *og = static_cast<bf16 *>(a.out);

    // State fragments: warp w owns rows 16 (w % 8) .. +15 and columns 64 (w / 8) .. +63.
    const int srow = 16 * (warp & 7), scol = 64 * (warp >> 3);
    float S[8][4];
    {
        const float *init = a.initial_state ? a.initial_state + (int64_t(seq) * H + head) * PK * PV : nullptr;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int row = srow + g8 + 8 * (e >> 1), col = scol + 8 * nt + 2 * tig + (e & 1);
                S[nt][e] = init ? init[row * PV + col] : 0.f;
            }
            const int col = scol + 8 * nt + 2 * tig;
            *reinterpret_cast<uint32_t *>(&s.s[srow + g8][col]) = pack_bf16(S[nt][0], S[nt][1]);
            *reinterpret_cast<uint32_t *>(&s.s[srow + g8 + 8][col]) = pack_bf16(S[nt][2], S[nt][3]);
        }
    }
    if (chunks > 0) stage_chunk(a, s.st[0], rec0, range.x, min(PC, range.y - range.x), qh, tid);
    asm volatile("cp.async.commit_group;\n" ::);
    // Chunk-output fragments: warp w owns rows 16 (w % 4) and columns 32 (w / 4) .. +31.
    const int orow = 16 * (warp & 3), ocol = 32 * (warp >> 2);

    for (int c = 0; c < chunks; ++c) {
        StateStage &st = s.st[c & 1];
        const int t0 = range.x + c * PC, n = min(PC, range.y - t0);
        if (c + 1 < chunks)
            stage_chunk(a, s.st[(c + 1) & 1], rec0 + int64_t(c + 1) * H * kRec, t0 + PC, min(PC, range.y - t0 - PC), qh, tid);
        asm volatile("cp.async.commit_group;\ncp.async.wait_group 1;\n" ::);
        __syncthreads();

        // ---- D = U - W S, O = diag(e^gam nq scale) Q S
        float D[4][4], O[4][4] = {};
        const int i0 = orow + g8, i1 = i0 + 8;
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
            const int col = ocol + 8 * nt + 2 * tig;
            const float2 u0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&st.u[i0][col]));
            const float2 u1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&st.u[i1][col]));
            D[nt][0] = u0.x;
            D[nt][1] = u0.y;
            D[nt][2] = u1.x;
            D[nt][3] = u1.y;
        }
#pragma unroll
        for (int ks = 0; ks < PK / 16; ++ks) {
            uint32_t aw[4], aq[4], b0[4], b1[4];
            load_a<kLd>(aw, st.w, orow, 16 * ks, lane);
            load_a<kLd>(aq, st.q, orow, 16 * ks, lane);
            load_b_kn<kLd>(b0, s.s, ocol, 16 * ks, lane);
            load_b_kn<kLd>(b1, s.s, ocol + 16, 16 * ks, lane);
            mma16816(D[0], aw, b0[0], b0[1]);
            mma16816(D[1], aw, b0[2], b0[3]);
            mma16816(D[2], aw, b1[0], b1[1]);
            mma16816(D[3], aw, b1[2], b1[3]);
            mma16816(O[0], aq, b0[0], b0[1]);
            mma16816(O[1], aq, b0[2], b0[3]);
            mma16816(O[2], aq, b1[0], b1[1]);
            mma16816(O[3], aq, b1[2], b1[3]);
        }
        {
            const float o0 = st.ro[i0], o1 = st.ro[i1], d0 = st.rd[i0], d1 = st.rd[i1];
#pragma unroll
            for (int nt = 0; nt < 4; ++nt) {
                const int col = ocol + 8 * nt + 2 * tig;
                O[nt][0] *= o0;
                O[nt][1] *= o0;
                O[nt][2] *= o1;
                O[nt][3] *= o1;
                *reinterpret_cast<uint32_t *>(&s.d[i0][col]) = pack_bf16(D[nt][0], D[nt][1]);
                *reinterpret_cast<uint32_t *>(&s.d[i1][col]) = pack_bf16(D[nt][2], D[nt][3]);
                *reinterpret_cast<uint32_t *>(&s.dt[i0][col]) = pack_bf16(d0 * D[nt][0], d0 * D[nt][1]);
                *reinterpret_cast<uint32_t *>(&s.dt[i1][col]) = pack_bf16(d1 * D[nt][2], d1 * D[nt][3]);
            }
        }
        __syncthreads();

        // ---- O += P D; store the chunk's outputs
#pragma unroll
        for (int ks = 0; ks < PC / 16; ++ks) {
            uint32_t ap[4], b0[4], b1[4];
            load_a<kLdP>(ap, st.p, orow, 16 * ks, lane);
            load_b_kn<kLd>(b0, s.d, ocol, 16 * ks, lane);
            load_b_kn<kLd>(b1, s.d, ocol + 16, 16 * ks, lane);
            mma16816(O[0], ap, b0[0], b0[1]);
            mma16816(O[1], ap, b0[2], b0[3]);
            mma16816(O[2], ap, b1[0], b1[1]);
            mma16816(O[3], ap, b1[2], b1[3]);
        }
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
            const int col = ocol + 8 * nt + 2 * tig;
            if (i0 < n)
                *reinterpret_cast<uint32_t *>(og + ((int64_t(t0) + i0) * H + head) * PV + col) = pack_bf16(O[nt][0], O[nt][1]);
            if (i1 < n)
                *reinterpret_cast<uint32_t *>(og + ((int64_t(t0) + i1) * H + head) * PV + col) = pack_bf16(O[nt][2], O[nt][3]);
        }

        // ---- S = e^gam_C S + K^T Dt, then its bf16 copy
        {
            const float dc = st.dc[0];
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
                for (int e = 0; e < 4; ++e) S[nt][e] *= dc;
            }
#pragma unroll
            for (int ks = 0; ks < PC / 16; ++ks) {
                uint32_t ak[4];
                load_a_t<kLd>(ak, st.k, srow, 16 * ks, lane);
#pragma unroll
                for (int np = 0; np < 4; ++np) {
                    uint32_t b[4];
                    load_b_kn<kLd>(b, s.dt, scol + 16 * np, 16 * ks, lane);
                    mma16816(S[2 * np], ak, b[0], b[1]);
                    mma16816(S[2 * np + 1], ak, b[2], b[3]);
                }
            }
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) {
                const int col = scol + 8 * nt + 2 * tig;
                *reinterpret_cast<uint32_t *>(&s.s[srow + g8][col]) = pack_bf16(S[nt][0], S[nt][1]);
                *reinterpret_cast<uint32_t *>(&s.s[srow + g8 + 8][col]) = pack_bf16(S[nt][2], S[nt][3]);
            }
        }
        __syncthreads();  // the state copy is complete; this stage is refilled next chunk
    }
    asm volatile("cp.async.wait_group 0;\n" ::);

    float *fin = a.final_state + (int64_t(seq) * H + head) * PK * PV;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
        const int col = scol + 8 * nt + 2 * tig;
        *reinterpret_cast<float2 *>(fin + (srow + g8) * PV + col) = make_float2(S[nt][0], S[nt][1]);
        *reinterpret_cast<float2 *>(fin + (srow + g8 + 8) * PV + col) = make_float2(S[nt][2], S[nt][3]);
    }
}

bool aligned_rows(const void *p, int64_t stride) {
    return (reinterpret_cast<uintptr_t>(p) & 15u) == 0 && (stride * 2) % 16 == 0;
}

int64_t max_chunks(int64_t tokens, int64_t seqs) { return (tokens + PC - 1) / PC + seqs; }

}  // namespace
}  // namespace sq

extern "C" int64_t sq_gdn_prefill_workspace_bytes(int32_t tokens, int32_t num_seqs, int32_t heads) {
    if (tokens < 0 || num_seqs < 0 || heads < 1) return -1;
    return sq::kOffsetsBytes(num_seqs) + sq::max_chunks(tokens, num_seqs) * heads * int64_t(sq::kRec);
}

extern "C" int32_t sq_gdn_prefill(const sq_prefill_args *args, sq_stream_t stream) {
    if (!args) return SQ_ERR_ARGUMENT;
    const sq_prefill_args &a = *args;
    if (a.num_seqs < 0 || a.tokens < 0 || a.heads < 1 || a.qk_heads < 1) return SQ_ERR_ARGUMENT;
    if (a.heads % a.qk_heads) return SQ_ERR_SHAPE;
    if (a.keys != sq::PK || a.values != sq::PV || a.io_dtype != SQ_BF16) return SQ_ERR_UNSUPPORTED;
    if (a.num_seqs == 0) return SQ_OK;
    if (!a.q || !a.k || !a.v || !a.g || !a.beta || !a.cu_seqlens || !a.final_state || !a.out || !a.workspace)
        return SQ_ERR_ARGUMENT;
    if (a.workspace_bytes < sq_gdn_prefill_workspace_bytes(a.tokens, a.num_seqs, a.heads)) return SQ_ERR_CAPACITY;
    if (a.q_stride < 0 || a.k_stride < 0 || a.v_stride < 0) return SQ_ERR_SHAPE;
    if (!sq::aligned_rows(a.q, a.q_stride) || !sq::aligned_rows(a.k, a.k_stride) || !sq::aligned_rows(a.v, a.v_stride) ||
        (reinterpret_cast<uintptr_t>(a.out) & 3u) || (reinterpret_cast<uintptr_t>(a.final_state) & 7u) ||
        (reinterpret_cast<uintptr_t>(a.workspace) & 255u))
        return SQ_ERR_SHAPE;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    int32_t *offsets = static_cast<int32_t *>(a.workspace);
    unsigned char *records = static_cast<unsigned char *>(a.workspace) + sq::kOffsetsBytes(a.num_seqs);
    sq::offsets_kernel<<<1, 1024, 0, s>>>(a, offsets);
    const int prep_smem = int(sizeof(sq::PrepSmem)), state_smem = int(sizeof(sq::StateSmem));
    if (cudaFuncSetAttribute(sq::prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, prep_smem) != cudaSuccess ||
        cudaFuncSetAttribute(sq::state_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, state_smem) != cudaSuccess)
        return SQ_ERR_CUDA;
    const int64_t chunks = sq::max_chunks(a.tokens, a.num_seqs);
    if (chunks > 0x7fffffff) return SQ_ERR_SHAPE;
    if (chunks > 0) sq::prep_kernel<<<dim3(unsigned(chunks), unsigned(a.heads)), 256, prep_smem, s>>>(a, offsets, records);
    sq::state_kernel<<<a.num_seqs * a.heads, 512, state_smem, s>>>(a, offsets, records);
    return cudaGetLastError() == cudaSuccess ? SQ_OK : SQ_ERR_CUDA;
}
