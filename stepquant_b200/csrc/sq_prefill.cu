// GDN chunked prefill (WY/UT form) on tensor cores.
//
// One 512-thread CTA per (sequence, value head) walks the sequence in 64-token
// chunks.  Within a chunk with cumulative log decay gam_i and normalisations
// nk, nq (applied in fp32 to exact bf16 products of the raw inputs):
//   L_ij = beta_i exp(gam_i - gam_j) nk_i nk_j (k_i . k_j)          (j < i)
//   P_ij = exp(gam_i - gam_j) nq_i scale nk_j (q_i . k_j)            (j <= i)
//   T    = (I + L)^-1       (fp32: 16x16 diagonal blocks by substitution,
//                            off-diagonal blocks T_rc = -T_rr sum_m L_rm T_mc)
//   W    = T diag(beta e^gam nk) K,   U = T diag(beta) V
//   D    = U - W S                    (the chunk's beta-scaled residuals)
//   O    = diag(e^gam nq scale) Q S + P D
//   S'   = e^gam_C S + K^T diag(e^(gam_C - gam) nk) D
// which equals the token-by-token recurrence of core.delta_step.  Every
// product is an mma.sync m16n8k16 bf16 tile with fp32 accumulation (operands
// staged in padded shared memory and read with ldmatrix); the state S lives
// in fp32 registers for the whole sequence and is copied to shared memory in
// bf16 as the operand of W S and Q S.  Padded tokens of the last chunk have
// beta = 0 and log decay 0, so they leave the state unchanged.
#include "sq_common.cuh"

namespace sq {
namespace {

constexpr int PC = 64;    // chunk length
constexpr int PK = 128;   // keys
constexpr int PV = 128;   // values
constexpr int kPT = 512;  // threads per CTA
constexpr int kLd = 136;  // bf16 row stride of 128-wide tiles (272 B: ldmatrix rows hit distinct banks)
constexpr int kLdP = 72;  // bf16 row stride of 64-wide tiles
constexpr int kLdF = 68;  // fp32 row stride of 64x64 tiles

using bf16 = __nv_bfloat16;

// Region shared by the phases of a chunk (byte offsets):
//   L, T, X (fp32 64x68 each)   at 0, 17408, 34816        -- the inverse
//   Tw, Tu (bf16 64x72)         at 0, 34816                -- not over T
//   D, Dt (bf16 64x136)         at 0, 17408                -- after W and U
constexpr int kRegion = 3 * PC * kLdF * 4;

struct PrefillSmem {
    bf16 q[PC][kLd];
    bf16 k[PC][kLd];
    bf16 v[PC][kLd];  // raw v; then -W
    bf16 s[PK][kLd];  // the state in bf16 (operand of W S and Q S)
    bf16 p[PC][kLdP];
    alignas(16) unsigned char region[kRegion];
    float gam[PC];
    float beta[PC];
    float nq[PC];
    float nk[PC];
};

__device__ __forceinline__ float (*tri_l(PrefillSmem &s))[kLdF] { return reinterpret_cast<float (*)[kLdF]>(s.region); }
__device__ __forceinline__ float (*tri_t(PrefillSmem &s))[kLdF] { return reinterpret_cast<float (*)[kLdF]>(s.region + PC * kLdF * 4); }
__device__ __forceinline__ float (*tri_x(PrefillSmem &s))[kLdF] { return reinterpret_cast<float (*)[kLdF]>(s.region + 2 * PC * kLdF * 4); }
__device__ __forceinline__ bf16 (*mat_tw(PrefillSmem &s))[kLdP] { return reinterpret_cast<bf16 (*)[kLdP]>(s.region); }
__device__ __forceinline__ bf16 (*mat_tu(PrefillSmem &s))[kLdP] { return reinterpret_cast<bf16 (*)[kLdP]>(s.region + 2 * PC * kLdF * 4); }
__device__ __forceinline__ bf16 (*mat_d(PrefillSmem &s))[kLd] { return reinterpret_cast<bf16 (*)[kLd]>(s.region); }
__device__ __forceinline__ bf16 (*mat_dt(PrefillSmem &s))[kLd] { return reinterpret_cast<bf16 (*)[kLd]>(s.region + PC * kLdF * 4); }

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

__global__ void __launch_bounds__(kPT, 1) prefill_kernel(sq_prefill_args a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    PrefillSmem &s = *reinterpret_cast<PrefillSmem *>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g8 = lane >> 2, tig = lane & 3;
    const int H = a.heads;
    const int seq = blockIdx.x / H, head = blockIdx.x % H;
    const int qh = head / (H / a.qk_heads);
    const int begin = max(0, min(a.cu_seqlens[seq], a.tokens));
    const int end = max(begin, min(a.cu_seqlens[seq + 1], a.tokens));
    const bf16 *qg = static_cast<const bf16 *>(a.q);
    const bf16 *kg = static_cast<const bf16 *>(a.k);
    const bf16 *vg = static_cast<const bf16 *>(a.v);
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
        }
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
            const int col = scol + 8 * nt + 2 * tig;
            *reinterpret_cast<uint32_t *>(&s.s[srow + g8][col]) = pack_bf16(S[nt][0], S[nt][1]);
            *reinterpret_cast<uint32_t *>(&s.s[srow + g8 + 8][col]) = pack_bf16(S[nt][2], S[nt][3]);
        }
    }
    // Chunk-output fragments: warp w owns rows 16 (w % 4) and columns 32 (w / 4) .. +31.
    const int orow = 16 * (warp & 3), ocol = 32 * (warp >> 2);

    for (int t0 = begin; t0 < end; t0 += PC) {
        const int n = min(PC, end - t0);
        // ---- load the chunk's raw q, k, v rows (zero rows past the end) and gates
        for (int idx = tid; idx < 3 * PC * 16; idx += kPT) {
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

        // ---- norms of q and k rows (4 threads per row), cumulative log decay
        {
            const int row = (tid >> 2) & 63, quarter = tid & 3;
            const bf16 *src = tid < 256 ? s.q[row] : s.k[row];
            float ss = 0.f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint4 w = *reinterpret_cast<const uint4 *>(src + quarter * 32 + j * 8);
                const __nv_bfloat162 *h2 = reinterpret_cast<const __nv_bfloat162 *>(&w);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f = __bfloat1622float2(h2[e]);
                    ss += f.x * f.x + f.y * f.y;
                }
            }
            ss += __shfl_xor_sync(0xffffffffu, ss, 1);
            ss += __shfl_xor_sync(0xffffffffu, ss, 2);
            const float nrm = a.normalize ? rsqrtf(ss + 1e-6f) : 1.f;
            if (quarter == 0) {
                if (tid < 256) s.nq[row] = nrm;
                else s.nk[row] = nrm;
            }
        }
        if (warp == 0) {
            // inclusive scan of the chunk's log decays (2 per lane)
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

        // ---- G = K K^T and H = Q K^T tiles -> L (fp32) and P (bf16)
        {
            const int tr = warp >> 2, tc = warp & 3;
            float (*L)[kLdF] = tri_l(s);
            if (tc <= tr) {
                float accG[2][4] = {}, accH[2][4] = {};
#pragma unroll
                for (int ks = 0; ks < PK / 16; ++ks) {
                    uint32_t ak[4], aq[4], b[4];
                    load_a<kLd>(ak, s.k, 16 * tr, 16 * ks, lane);
                    load_a<kLd>(aq, s.q, 16 * tr, 16 * ks, lane);
                    load_b_nk<kLd>(b, s.k, 16 * tc, 16 * ks, lane);
                    mma16816(accG[0], ak, b[0], b[1]);
                    mma16816(accG[1], ak, b[2], b[3]);
                    mma16816(accH[0], aq, b[0], b[1]);
                    mma16816(accH[1], aq, b[2], b[3]);
                }
#pragma unroll
                for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int i = 16 * tr + g8 + 8 * (e >> 1), j = 16 * tc + 8 * nt + 2 * tig + (e & 1);
                        const float dec = j <= i ? expf(s.gam[i] - s.gam[j]) : 0.f;
                        L[i][j] = j < i ? s.beta[i] * dec * s.nk[i] * s.nk[j] * accG[nt][e] : 0.f;
                        s.p[i][j] = __float2bfloat16_rn(dec * s.nq[i] * a.scale * s.nk[j] * accH[nt][e]);
                    }
                }
            } else {
#pragma unroll
                for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int i = 16 * tr + g8 + 8 * (e >> 1), j = 16 * tc + 8 * nt + 2 * tig + (e & 1);
                        s.p[i][j] = __float2bfloat16_rn(0.f);
                    }
                }
            }
        }
        __syncthreads();

        // ---- T = (I + L)^-1: diagonal blocks by substitution, then block rows 1..3
        {
            float (*L)[kLdF] = tri_l(s);
            float (*T)[kLdF] = tri_t(s);
            float (*X)[kLdF] = tri_x(s);
            if (warp < 4 && lane < 16) {
                const int b = 16 * warp, m = lane;
                float t[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    float val = i == m ? 1.f : 0.f;
#pragma unroll
                    for (int j = 0; j < i; ++j) val -= L[b + i][b + j] * t[j];
                    t[i] = val;
                    T[b + i][b + m] = val;
                }
            } else if (warp >= 4) {
                // zero the blocks above the diagonal
                for (int e = tid - 128; e < 6 * 256; e += kPT - 128) {
                    const int blk = e >> 8, i = (e >> 4) & 15, m = e & 15;
                    const int r = blk < 3 ? 0 : blk < 5 ? 1 : 2;
                    const int c = blk < 3 ? blk + 1 : blk < 5 ? blk - 1 : 3;
                    T[16 * r + i][16 * c + m] = 0.f;
                }
            }
            __syncthreads();
            for (int r = 1; r < 4; ++r) {
                for (int e = tid; e < r * 256; e += kPT) {
                    const int c = e >> 8, i = (e >> 4) & 15, m = e & 15;
                    float x = 0.f;
                    for (int j = 16 * c; j < 16 * r; ++j) x += L[16 * r + i][j] * T[j][16 * c + m];
                    X[16 * r + i][16 * c + m] = x;
                }
                __syncthreads();
                for (int e = tid; e < r * 256; e += kPT) {
                    const int c = e >> 8, i = (e >> 4) & 15, m = e & 15;
                    float t = 0.f;
#pragma unroll
                    for (int j = 0; j < 16; ++j) t -= T[16 * r + i][16 * r + j] * X[16 * r + j][16 * c + m];
                    T[16 * r + i][16 * c + m] = t;
                }
                __syncthreads();
            }
        }

        // ---- Tw = T diag(beta e^gam nk), Tu = T diag(beta) in bf16
        {
            float (*T)[kLdF] = tri_t(s);
            bf16 (*Tw)[kLdP] = mat_tw(s);
            bf16 (*Tu)[kLdP] = mat_tu(s);
            for (int e = tid; e < PC * PC; e += kPT) {
                const int i = e >> 6, j = e & 63;
                const float t = T[i][j];
                Tw[i][j] = __float2bfloat16_rn(t * (s.beta[j] * expf(s.gam[j]) * s.nk[j]));
                Tu[i][j] = __float2bfloat16_rn(t * s.beta[j]);
            }
        }
        __syncthreads();

        // ---- W = Tw K, U = Tu V (rows 16 (w % 4), columns 32 (w / 4) .. +31)
        float D[4][4] = {}, W[4][4] = {};
        {
            bf16 (*Tw)[kLdP] = mat_tw(s);
            bf16 (*Tu)[kLdP] = mat_tu(s);
#pragma unroll
            for (int ks = 0; ks < PC / 16; ++ks) {
                uint32_t aw[4], au[4], bk0[4], bk1[4], bv0[4], bv1[4];
                load_a<kLdP>(aw, Tw, orow, 16 * ks, lane);
                load_a<kLdP>(au, Tu, orow, 16 * ks, lane);
                load_b_kn<kLd>(bk0, s.k, ocol, 16 * ks, lane);
                load_b_kn<kLd>(bk1, s.k, ocol + 16, 16 * ks, lane);
                load_b_kn<kLd>(bv0, s.v, ocol, 16 * ks, lane);
                load_b_kn<kLd>(bv1, s.v, ocol + 16, 16 * ks, lane);
                mma16816(W[0], aw, bk0[0], bk0[1]);
                mma16816(W[1], aw, bk0[2], bk0[3]);
                mma16816(W[2], aw, bk1[0], bk1[1]);
                mma16816(W[3], aw, bk1[2], bk1[3]);
                mma16816(D[0], au, bv0[0], bv0[1]);
                mma16816(D[1], au, bv0[2], bv0[3]);
                mma16816(D[2], au, bv1[0], bv1[1]);
                mma16816(D[3], au, bv1[2], bv1[3]);
            }
        }
        __syncthreads();
        // -W into the v tile (v is no longer needed)
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
            const int col = ocol + 8 * nt + 2 * tig;
            *reinterpret_cast<uint32_t *>(&s.v[orow + g8][col]) = pack_bf16(-W[nt][0], -W[nt][1]);
            *reinterpret_cast<uint32_t *>(&s.v[orow + g8 + 8][col]) = pack_bf16(-W[nt][2], -W[nt][3]);
        }
        __syncthreads();

        // ---- D = U - W S, O = diag(e^gam nq scale) Q S
        float O[4][4] = {};
#pragma unroll
        for (int ks = 0; ks < PK / 16; ++ks) {
            uint32_t aw[4], aq[4], b0[4], b1[4];
            load_a<kLd>(aw, s.v, orow, 16 * ks, lane);
            load_a<kLd>(aq, s.q, orow, 16 * ks, lane);
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
        const float gC = s.gam[PC - 1];
        {
            bf16 (*Dm)[kLd] = mat_d(s);
            bf16 (*Dt)[kLd] = mat_dt(s);
            const int i0 = orow + g8, i1 = i0 + 8;
            const float o0 = expf(s.gam[i0]) * s.nq[i0] * a.scale, o1 = expf(s.gam[i1]) * s.nq[i1] * a.scale;
            const float d0 = expf(gC - s.gam[i0]) * s.nk[i0], d1 = expf(gC - s.gam[i1]) * s.nk[i1];
#pragma unroll
            for (int nt = 0; nt < 4; ++nt) {
                const int col = ocol + 8 * nt + 2 * tig;
                O[nt][0] *= o0;
                O[nt][1] *= o0;
                O[nt][2] *= o1;
                O[nt][3] *= o1;
                *reinterpret_cast<uint32_t *>(&Dm[i0][col]) = pack_bf16(D[nt][0], D[nt][1]);
                *reinterpret_cast<uint32_t *>(&Dm[i1][col]) = pack_bf16(D[nt][2], D[nt][3]);
                *reinterpret_cast<uint32_t *>(&Dt[i0][col]) = pack_bf16(d0 * D[nt][0], d0 * D[nt][1]);
                *reinterpret_cast<uint32_t *>(&Dt[i1][col]) = pack_bf16(d1 * D[nt][2], d1 * D[nt][3]);
            }
        }
        __syncthreads();

        // ---- O += P D; store the chunk's outputs
        {
            bf16 (*Dm)[kLd] = mat_d(s);
#pragma unroll
            for (int ks = 0; ks < PC / 16; ++ks) {
                uint32_t ap[4], b0[4], b1[4];
                load_a<kLdP>(ap, s.p, orow, 16 * ks, lane);
                load_b_kn<kLd>(b0, Dm, ocol, 16 * ks, lane);
                load_b_kn<kLd>(b1, Dm, ocol + 16, 16 * ks, lane);
                mma16816(O[0], ap, b0[0], b0[1]);
                mma16816(O[1], ap, b0[2], b0[3]);
                mma16816(O[2], ap, b1[0], b1[1]);
                mma16816(O[3], ap, b1[2], b1[3]);
            }
            const int i0 = orow + g8, i1 = i0 + 8;
#pragma unroll
            for (int nt = 0; nt < 4; ++nt) {
                const int col = ocol + 8 * nt + 2 * tig;
                if (i0 < n)
                    *reinterpret_cast<uint32_t *>(og + ((int64_t(t0) + i0) * H + head) * PV + col) = pack_bf16(O[nt][0], O[nt][1]);
                if (i1 < n)
                    *reinterpret_cast<uint32_t *>(og + ((int64_t(t0) + i1) * H + head) * PV + col) = pack_bf16(O[nt][2], O[nt][3]);
            }
        }

        // ---- S = e^gam_C S + K^T Dt (fp32 accumulators), then its bf16 copy
        {
            bf16 (*Dt)[kLd] = mat_dt(s);
            const float dc = expf(gC);
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
                for (int e = 0; e < 4; ++e) S[nt][e] *= dc;
            }
#pragma unroll
            for (int ks = 0; ks < PC / 16; ++ks) {
                uint32_t ak[4];
                load_a_t<kLd>(ak, s.k, srow, 16 * ks, lane);
#pragma unroll
                for (int np = 0; np < 4; ++np) {
                    uint32_t b[4];
                    load_b_kn<kLd>(b, Dt, scol + 16 * np, 16 * ks, lane);
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
        __syncthreads();  // the chunk's tiles are rewritten by the next load
    }

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

}  // namespace
}  // namespace sq

extern "C" int32_t sq_gdn_prefill(const sq_prefill_args *args, sq_stream_t stream) {
    if (!args) return SQ_ERR_ARGUMENT;
    const sq_prefill_args &a = *args;
    if (a.num_seqs < 0 || a.tokens < 0 || a.heads < 1 || a.qk_heads < 1) return SQ_ERR_ARGUMENT;
    if (a.heads % a.qk_heads) return SQ_ERR_SHAPE;
    if (a.keys != sq::PK || a.values != sq::PV || a.io_dtype != SQ_BF16) return SQ_ERR_UNSUPPORTED;
    if (a.num_seqs == 0) return SQ_OK;
    if (!a.q || !a.k || !a.v || !a.g || !a.beta || !a.cu_seqlens || !a.final_state || !a.out) return SQ_ERR_ARGUMENT;
    if (a.q_stride < 0 || a.k_stride < 0 || a.v_stride < 0) return SQ_ERR_SHAPE;
    if (!sq::aligned_rows(a.q, a.q_stride) || !sq::aligned_rows(a.k, a.k_stride) || !sq::aligned_rows(a.v, a.v_stride) ||
        (reinterpret_cast<uintptr_t>(a.out) & 3u) || (reinterpret_cast<uintptr_t>(a.final_state) & 7u))
        return SQ_ERR_SHAPE;
    const int smem = int(sizeof(sq::PrefillSmem));
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t err = cudaFuncSetAttribute(sq::prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (err != cudaSuccess) return SQ_ERR_CUDA;
    sq::prefill_kernel<<<a.num_seqs * a.heads, sq::kPT, smem, s>>>(a);
    return cudaGetLastError() == cudaSuccess ? SQ_OK : SQ_ERR_CUDA;
}
