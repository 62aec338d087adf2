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
// factors -- into a workspace record (bf16 products on tcgen05, fp32 inverse);
// state_kernel (one CTA per sequence and value head) walks the chunks in order
// with the 128x128 state in tensor memory, on tcgen05 (see its comment).
// Padded tokens of a last partial chunk have beta = 0 and log decay 0, so they
// leave the state unchanged.
#include "sq_common.cuh"

namespace sq {
namespace {

constexpr int PC = 64;    // chunk length
constexpr int PK = 128;   // keys
constexpr int PV = 128;   // values
constexpr int kLdF = 68;  // fp32 row stride of 64x64 tiles

using bf16 = __nv_bfloat16;

// Workspace record of one (chunk, value head), byte offsets.  -W and P are
// stored as the state kernel's shared-memory operand tiles (128-byte swizzle).
constexpr int kRecW = 0;                     // -W   bf16 [64][128] K-major tile
constexpr int kRecP = kRecW + PC * PK * 2;    // P    bf16 [64][64]  K-major tile
constexpr int kRecU = kRecP + PC * PC * 2;    // U    bf16 [64][128] row-major
constexpr int kRecRo = kRecU + PC * PV * 2;   // e^gam nq scale      fp32 [64]
constexpr int kRecRd = kRecRo + PC * 4;       // e^(gam_C - gam) nk  fp32 [64]
constexpr int kRecDc = kRecRd + PC * 4;       // e^gam_C             fp32 (16 bytes)
constexpr int kRec = (kRecDc + 16 + 255) / 256 * 256;
constexpr int kOffsetsBytes(int seqs) { return (4 * (seqs + 1) + 255) / 256 * 256; }
constexpr int64_t kChunkTabBytes(int64_t chunks) { return (8 * chunks + 255) / 256 * 256; }

__device__ __forceinline__ unsigned smem_addr(const void *p) { return static_cast<unsigned>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ void cp16(void *smem, const void *gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_addr(smem)), "l"(gmem));
}

__device__ __forceinline__ uint32_t tf32_bits(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;\n" : "=r"(r) : "f"(x));
    return r;
}
// d += a (16x8, tf32, row-major fragment) * b (8x8, tf32, column fragment); fp32 accumulators.
__device__ __forceinline__ void mma1688_tf32(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&v);
}

// Byte offset of element (row, k) of a bf16 K-major operand tile with `rows`
// rows under the 128-byte swizzle: K in atoms of 64 elements (rows * 128 bytes
// each), rows in groups of 8 (1024 bytes), 16-byte chunk c of row r stored at
// chunk c ^ (r % 8).
__device__ __forceinline__ uint32_t sw128(int row, int k, int rows) {
    const int kin = k & 63;
    return (k >> 6) * (rows * 128) + (row >> 3) * 1024 + (row & 7) * 128 + ((((kin >> 3) ^ (row & 7))) << 4) + (kin & 7) * 2;
}
// The same for an MN-major tile with `krows` K rows: N in groups of 64
// elements (krows * 128 bytes apart), K rows in groups of 8 (1024 bytes).
__device__ __forceinline__ uint32_t sw128_mn(int kk, int n, int krows) {
    const int nin = n & 63;
    return (n >> 6) * (krows / 8) * 1024 + (kk >> 3) * 1024 + (kk & 7) * 128 + ((((nin >> 3) ^ (kk & 7))) << 4) + (nin & 7) * 2;
}

// Token range of sequence n, clamped to [0, tokens).
__device__ __forceinline__ int2 seq_range(const sq_prefill_args &a, int n) {
    const int b = max(0, min(a.cu_seqlens[n], a.tokens));
    return make_int2(b, max(b, min(a.cu_seqlens[n + 1], a.tokens)));
}

// offsets[n] = number of chunks of the sequences before n (offsets[seqs] = all),
// and for every chunk its first token and length (chunk_tab).
__global__ void __launch_bounds__(1024) offsets_kernel(sq_prefill_args a, int32_t *offsets, int2 *chunk_tab) {
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
        for (int t = r.x; t < r.y; t += PC) chunk_tab[before++] = make_int2(t, min(PC, r.y - t));
    }
    if (threadIdx.x == 0) offsets[a.num_seqs] = warp_total[31];
}

// acc (a 16x16 block as two 16x8 tf32 accumulator tiles) += A[ar0.., ac0..] B[br0.., bc0..]
// over a 16-deep k range (two m16n8k8 steps); fp32 operands rounded to tf32.
__device__ __forceinline__ void mma_block16(float (&acc)[2][4], const float (*A)[kLdF], int ar0, int ac0,
                                            const float (*B)[kLdF], int br0, int bc0, int g8, int tig) {
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
        uint32_t af[4];
        af[0] = tf32_bits(A[ar0 + g8][ac0 + 8 * kk + tig]);
        af[1] = tf32_bits(A[ar0 + g8 + 8][ac0 + 8 * kk + tig]);
        af[2] = tf32_bits(A[ar0 + g8][ac0 + 8 * kk + tig + 4]);
        af[3] = tf32_bits(A[ar0 + g8 + 8][ac0 + 8 * kk + tig + 4]);
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
            const uint32_t b0 = tf32_bits(B[br0 + 8 * kk + tig][bc0 + 8 * nt + g8]);
            const uint32_t b1 = tf32_bits(B[br0 + 8 * kk + tig + 4][bc0 + 8 * nt + g8]);
            mma1688_tf32(acc[nt], af, b0, b1);
        }
    }
}
__device__ __forceinline__ void store_block16(const float (&acc)[2][4], float (*dst)[kLdF], int g8, int tig) {
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
        const int col = 8 * nt + 2 * tig;
        dst[g8][col] = acc[nt][0];
        dst[g8][col + 1] = acc[nt][1];
        dst[g8 + 8][col] = acc[nt][2];
        dst[g8 + 8][col + 1] = acc[nt][3];
    }
}

// ---------------------------------------------------------------------------
// state_kernel: one 512-thread CTA per (sequence, value head), on tcgen05.
// The transposed products keep every accumulator at M = 128 rows = the value
// columns: warp w reads TMEM lanes 32 (w % 4) .. +31 (value columns) and the
// quarter w / 4 of each accumulator's columns.  TMEM columns (fp32):
//   S^T [0, 128)   the state                     S^T += Dt^T K      (N = 128)
//   D^T [128, 192) the chunk residuals           D^T  = S^T (-W)^T  (N = 64), + U^T
//   O1^T [192,256) (Q S)^T                       O1^T = S^T Q^T     (N = 64)
//   O2^T [256,320) (P D)^T                       O2^T = D^T P^T     (N = 64)
// Odd chunks keep D^T in [320, 384) and O1^T in [384, 448), so the next
// chunk's D^T and O1^T products run while this chunk's outputs are read.
// Operands are bf16 in shared memory, 128-byte swizzled: S^T, D^T, Dt^T as
// K-major A tiles written by the threads; -W, P (from the record, bulk copies),
// raw q (cp.async) as K-major B tiles; raw k as an MN-major B tile.  One
// thread issues the MMAs; tcgen05.commit arrives on an mbarrier the others
// wait on (bounded waits: a CTA that gives up sets SQ_STATUS_TIMEOUT and
// leaves after freeing its tensor memory).
// ---------------------------------------------------------------------------
constexpr int kTmemCols = 512;
constexpr int kColS = 0, kColD = 128, kColO1 = 192, kColO2 = 256, kColD1 = 320, kColO11 = 384;
constexpr uint32_t kWaitLimit = 1u << 22;

struct TcStage {                 // offsets are multiples of 1024 (swizzle atoms)
    unsigned char w[16384];      // -W   [t][k]  K-major
    unsigned char p[8192];       // P    [i][j]  K-major
    unsigned char u[16384];      // U    [t][v]  bf16 row-major
    unsigned char q[16384];      // q    [t][k]  K-major
    unsigned char k[16384];      // k    [t][k]  MN-major (N = k)
    float ro[PC];                // e^gam nq scale
    float rd[PC];                // e^(gam_C - gam) nk
    float dc[4];                 // e^gam_C
    unsigned char pad[1024 - 528];
};
struct TcSmem {
    TcStage st[2];
    unsigned char sb[32768];     // S^T bf16 [v][k]
    unsigned char dm[16384];     // D^T bf16 [v][t]
    unsigned char dtm[16384];    // Dt^T bf16 [v][t]
};

__device__ __forceinline__ uint64_t sdesc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return uint64_t((addr >> 4) & 0x3FFF) | (uint64_t((lbo >> 4) & 0x3FFF) << 16) | (uint64_t((sbo >> 4) & 0x3FFF) << 32) |
           (1ull << 46) | (2ull << 61);  // sm100 descriptor version 1, 128-byte swizzle
}
// bf16 x bf16 -> fp32, M = 128, A K-major, B K-major (0) or MN-major (1)
__device__ __forceinline__ uint32_t idesc_bf16(int n, int b_mn) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(b_mn) << 16) | (uint32_t(n >> 3) << 17) | (uint32_t(128 >> 4) << 24);
}
__device__ __forceinline__ void umma(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
    asm volatile("{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\ntcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
                 :: "r"(d), "l"(a), "l"(b), "r"(id), "r"(acc));
}
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" :: "r"(smem_addr(bar)));
}
__device__ __forceinline__ bool bar_wait(uint64_t *bar, uint32_t parity) {
    uint32_t done = 0;
    for (uint32_t it = 0; it < kWaitLimit && !done; ++it)
        asm volatile("{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}\n"
                     : "=r"(done) : "r"(smem_addr(bar)), "r"(parity));
    return done != 0;
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void proxy_fence() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }

#define SQ_R8(i) "=r"(r[i]), "=r"(r[i + 1]), "=r"(r[i + 2]), "=r"(r[i + 3]), "=r"(r[i + 4]), "=r"(r[i + 5]), "=r"(r[i + 6]), "=r"(r[i + 7])
#define SQ_W8(i) "r"(r[i]), "r"(r[i + 1]), "r"(r[i + 2]), "r"(r[i + 3]), "r"(r[i + 4]), "r"(r[i + 5]), "r"(r[i + 6]), "r"(r[i + 7])
// 32 consecutive fp32 columns of this thread's lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&out)[32]) {
    uint32_t r[32];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                 "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
                 : SQ_R8(0), SQ_R8(8), SQ_R8(16), SQ_R8(24) : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) out[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&in)[32]) {
    uint32_t r[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(in[i]);
    asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
                 "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n"
                 :: "r"(taddr), SQ_W8(0), SQ_W8(8), SQ_W8(16), SQ_W8(24) : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&out)[16]) {
    uint32_t r[16];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
                 : SQ_R8(0), SQ_R8(8) : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) out[i] = __uint_as_float(r[i]);
}
#undef SQ_R8
#undef SQ_W8

// Write N fp32 values (columns c0 .. c0 + N - 1 of row `row`) as bf16 into a K-major SW128 tile.
template <int N>
__device__ __forceinline__ void put_row(unsigned char *tile, int rows, int row, int c0, const float (&x)[N], float scale = 1.f) {
#pragma unroll
    for (int j = 0; j < N / 8; ++j) {
        uint4 w;
        w.x = pack_bf16(scale * x[8 * j], scale * x[8 * j + 1]);
        w.y = pack_bf16(scale * x[8 * j + 2], scale * x[8 * j + 3]);
        w.z = pack_bf16(scale * x[8 * j + 4], scale * x[8 * j + 5]);
        w.w = pack_bf16(scale * x[8 * j + 6], scale * x[8 * j + 7]);
        *reinterpret_cast<uint4 *>(tile + sw128(row, c0 + 8 * j, rows)) = w;
    }
}

// Copies of chunk (t0, n rows) into a stage: the record by three bulk copies
// completing on `bar` (issued by thread 0), raw q and k rows by cp.async.
__device__ __forceinline__ void tc_stage(const sq_prefill_args &a, TcStage &st, uint64_t *bar, const unsigned char *rec,
                                         int t0, int n, int qh, int tid) {
    if (tid == 0) {
        const uint32_t bytes = 16384 + 8192 + 16384 + 528;
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" :: "r"(smem_addr(bar)), "r"(bytes) : "memory");
        const unsigned char *src[4] = {rec + kRecW, rec + kRecP, rec + kRecU, rec + kRecRo};
        void *dst[4] = {st.w, st.p, st.u, st.ro};
        const uint32_t len[4] = {16384, 8192, 16384, 528};
#pragma unroll
        for (int i = 0; i < 4; ++i)
            asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n"
                         :: "r"(smem_addr(dst[i])), "l"(src[i]), "r"(len[i]), "r"(smem_addr(bar)) : "memory");
    }
    const bf16 *qg = static_cast<const bf16 *>(a.q), *kg = static_cast<const bf16 *>(a.k);
    for (int idx = tid; idx < 2 * PC * 16; idx += 512) {
        const int which = idx >> 10, row = (idx >> 4) & 63, piece = idx & 15;
        unsigned char *dst = which == 0 ? st.q + sw128(row, 8 * piece, PC) : st.k + sw128_mn(row, 8 * piece, PC);
        if (row < n) {
            const int64_t t = t0 + row;
            cp16(dst, (which == 0 ? qg + t * a.q_stride : kg + t * a.k_stride) + int64_t(qh) * PK + piece * 8);
        } else {
            *reinterpret_cast<uint4 *>(dst) = make_uint4(0u, 0u, 0u, 0u);
        }
    }
}

// ---------------------------------------------------------------------------
// prep_kernel: one 256-thread CTA per (chunk, value head): the chunk's WY/UT
// transform.  Its bf16 products run on tcgen05 with fp32 accumulators in
// tensor memory (128 columns; three CTAs per SM):
//   [K; Q] K^T -> columns [0, 64), lanes 0-63 = G = K K^T, lanes 64-127 = Q K^T
//   W^T = K^T Tw^T -> columns [0, 64)      (lane = key, column = token)
//   U^T = V^T Tu^T -> columns [64, 128)    (lane = value, column = token)
// q and k are staged as one 128-row 128-byte-swizzled tile (k rows 0-63, q
// rows 64-127): K-major as the A operand of [K; Q] K^T and as its B operand
// (the first 64 rows), and, being [token][key] with keys contiguous, the same
// bytes are the MN-major A operand K^T.  T = (I + L)^-1 stays in fp32 (16x16
// blocks: substitution on the diagonal, tf32 mma.sync below it); Tw and Tu go
// into the q rows of the tile once the Gram product has read them, raw v into
// the space of L once T is complete.  Waits on the MMAs are bounded: a CTA
// that gives up sets SQ_STATUS_TIMEOUT and leaves after freeing its columns.
// ---------------------------------------------------------------------------
constexpr int kPrepCols = 128;

struct PrepSmem {
    unsigned char qk[32768];  // SW128, 128 rows x 128 keys: k rows 0-63, q rows 64-127; then Tw, Tu
    union {
        float l[PC][kLdF];       // L below the diagonal; the block products X_rc above it (block (c, r))
        unsigned char v[16384];  // raw v [t][v], SW128 (MN-major A operand of V^T), once T is complete
    } lv;
    float t[PC][kLdF];  // T
    float gam[PC];
    float beta[PC];
    float nq[PC];
    float nk[PC];
    float fw[PC];  // beta e^gam nk: column factors of Tw
    uint64_t bar;  // tcgen05.commit of the MMAs (two phases)
    uint32_t tmem_slot;
    int abort_flag;
};
constexpr int kPrepSmemBytes = int(sizeof(PrepSmem)) + 1024;  // + alignment of the swizzled tiles
constexpr int kTwOff = 8192, kTuOff = 16384 + 8192;             // q rows of key atoms 0 and 1: 64x64 K-major tiles

__device__ __forceinline__ uint32_t idesc_bf16_ab(int n, int a_mn, int b_mn) {
    return idesc_bf16(n, b_mn) | (uint32_t(a_mn) << 15);
}

__global__ void __launch_bounds__(256, 3) prep_kernel(sq_prefill_args a, const int32_t *offsets,
                                                      const int2 *chunk_tab, unsigned char *records) {
    extern __shared__ unsigned char smem_raw[];
    PrepSmem &s = *reinterpret_cast<PrepSmem *>(smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g8 = lane >> 2, tig = lane & 3;
    // One CTA per (chunk, qk head): q, k, their norms and [K; Q] K^T serve
    // the qk head's R = H / HK value heads, which the CTA takes in turn.
    const int H = a.heads, HK = a.qk_heads, R = H / HK;
    const int chunk = blockIdx.x / HK, qh = blockIdx.x - chunk * HK;
    const int total = offsets[a.num_seqs];
    const int2 ci = chunk_tab[chunk];  // read beside the total (entries past it are unset)
    if (chunk >= total) return;
    const int t0 = ci.x, n = ci.y;
    unsigned char *tw = s.qk + kTwOff, *tu = s.qk + kTuOff;

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" :: "r"(smem_addr(&s.tmem_slot)), "r"(kPrepCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n");
    }
    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" :: "r"(smem_addr(&s.bar)));
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        s.abort_flag = 0;
    }
    // ---- raw q, k rows of the chunk (zero rows past the end), gates
    {
        const bf16 *qg = static_cast<const bf16 *>(a.q), *kg = static_cast<const bf16 *>(a.k);
        for (int idx = tid; idx < 2 * PC * 16; idx += 256) {
            const int which = idx >> 10, row = (idx >> 4) & 63, piece = idx & 15;
            unsigned char *dst = s.qk + sw128(which == 0 ? PC + row : row, 8 * piece, 2 * PC);
            if (row < n) {
                const int64_t t = t0 + row;
                const bf16 *src = which == 0 ? qg + t * a.q_stride + int64_t(qh) * PK : kg + t * a.k_stride + int64_t(qh) * PK;
                cp16(dst, src + piece * 8);
            } else {
                *reinterpret_cast<uint4 *>(dst) = make_uint4(0u, 0u, 0u, 0u);
            }
        }
        if (tid < PC) {
            const bool live = tid < n;
            const int64_t gi = (int64_t(t0) + tid) * H + qh * R;
            s.gam[tid] = live ? a.g[gi] : 0.f;
            s.beta[tid] = live ? a.beta[gi] : 0.f;
        }
        asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;\n" ::: "memory");
    }
    proxy_fence();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s.tmem_slot;
    const uint32_t tlane = uint32_t(32 * (warp & 3)) << 16;  // this warp's TMEM lane quarter
    const int cq = warp >> 2;                                // and column half of each 64-column accumulator
    // ---- [K; Q] K^T on the tensor cores while the norms and the decay scan run
    // (issued from the last warp: warp 0 runs the scan)
    constexpr int kIssuer = 224;
    if (tid == kIssuer) {
        const uint32_t qk = smem_addr(s.qk), id = idesc_bf16(PC, 0);
#pragma unroll
        for (int ks = 0; ks < PK / 16; ++ks) {
            const uint32_t off = (ks >> 2) * 16384 + (ks & 3) * 32;
            umma(tmem, sdesc(qk + off, 16, 1024), sdesc(qk + off, 16, 1024), id, ks > 0);
        }
        umma_commit(&s.bar);
    }
    // norms of the q and k rows (2 threads per row), cumulative log decay
    {
        const int row = (tid >> 1) & 63, half = tid & 1;
        const int r = tid < 128 ? PC + row : row;
        const unsigned char *base = s.qk + half * 16384 + (r >> 3) * 1024 + (r & 7) * 128;
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint4 w = *reinterpret_cast<const uint4 *>(base + ((j ^ (r & 7)) << 4));
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
    uint32_t phase = 0;  // completed phases of s.bar: [K; Q] K^T, then W^T and U^T of each head
#pragma unroll 1
    for (int hr = 0; hr < R; ++hr) {
    const int head = qh * R + hr;
    unsigned char *rec = records + (int64_t(chunk) * H + head) * kRec;
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
    if (tid < PC) s.fw[tid] = s.beta[tid] * expf(s.gam[tid]) * s.nk[tid];
    if (hr == 0) {
        if (!bar_wait(&s.bar, 0)) s.abort_flag = 1;
        phase = 1;
    }
    tc_fence_after();
    // ---- L (fp32, from the G lanes) and P (bf16 into the record, from the Q K^T lanes).
    // A warp covers rows 32 (w % 2) .. +31 and columns 32 (w / 4) .. +31: the
    // quarter above the diagonal (rows 0-31, columns 32-63) is zero in P and
    // never read in L (the inverse reads L below the diagonal only).
    {
        const int r = 32 * (warp & 3) + lane, i = r & 63;
        const bool zero = 32 * cq > (i | 31);  // warp-uniform; L is not read there, P is written as zeros
        const float gi = s.gam[i];
        const float fi = r < PC ? s.beta[i] * s.nk[i] : s.nq[i] * a.scale;
#pragma unroll 1
        for (int half = 0; half < 2; ++half) {
            const int c0 = 32 * cq + 16 * half;
            float x[16], y[16];  // y: L (j < i) or P (j <= i)
            if (!zero) tmem_ld16(tmem + tlane + c0, x);
#pragma unroll
            for (int j4 = 0; j4 < 4; ++j4) {
                const float4 g4 = *reinterpret_cast<const float4 *>(&s.gam[c0 + 4 * j4]);
                const float4 n4 = *reinterpret_cast<const float4 *>(&s.nk[c0 + 4 * j4]);
                const float gj[4] = {g4.x, g4.y, g4.z, g4.w}, nkj[4] = {n4.x, n4.y, n4.z, n4.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int j = c0 + 4 * j4 + e;
                    const bool keep = !zero && (r < PC ? j < i : j <= i);
                    y[4 * j4 + e] = keep ? fi * (__expf(gi - gj[e]) * nkj[e]) * x[4 * j4 + e] : 0.f;
                }
            }
            if (r < PC) {
                if (!zero) {
                    float *lrow = &s.lv.l[i][c0];
#pragma unroll
                    for (int j4 = 0; j4 < 4; ++j4)
                        *reinterpret_cast<float4 *>(lrow + 4 * j4) =
                            make_float4(y[4 * j4], y[4 * j4 + 1], y[4 * j4 + 2], y[4 * j4 + 3]);
                }
            } else {
#pragma unroll
                for (int j8 = 0; j8 < 2; ++j8) {
                    const float *yy = y + 8 * j8;
                    *reinterpret_cast<uint4 *>(rec + kRecP + sw128(i, c0 + 8 * j8, PC)) =
                        make_uint4(pack_bf16(yy[0], yy[1]), pack_bf16(yy[2], yy[3]), pack_bf16(yy[4], yy[5]), pack_bf16(yy[6], yy[7]));
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();

    // ---- T = (I + L)^-1 in fp32: 16x16 diagonal blocks by substitution, then
    // the blocks below them on tensor cores (tf32); then Tw = T diag(beta e^gam nk)
    // and Tu = T diag(beta) in bf16 (K-major tiles in the q rows).
    if (warp < 4 && lane < 16) {
        const int b = 16 * warp, m = lane;
        float t[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            float val = i == m ? 1.f : 0.f;
#pragma unroll
            for (int j = 0; j < i; ++j) val -= s.lv.l[b + i][b + j] * t[j];
            t[i] = val;
            s.t[b + i][b + m] = val;
        }
    }
    __syncthreads();
    // Blocks below the diagonal as a blocked inverse in two stages:
    //   A: T10 = -T11 (L10 T00) (warp 0) and T32 = -T33 (L32 T22) (warp 1);
    //   B: T[2:4, 0:2] = -T[2:4, 2:4] (L[2:4, 0:2] T[0:2, 0:2]), one block per warp.
    // The block products X are kept in free blocks above L's diagonal.
    {
        float (*L)[kLdF] = s.lv.l;
        float (*T)[kLdF] = s.t;
        auto above = [&](int r, int c) { return reinterpret_cast<float (*)[kLdF]>(&L[16 * r][16 * c]); };
        auto finish = [&](int r, int c, const float (&Y)[2][4]) {  // T_rc = -Y, with its Tw and Tu blocks
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int i = 16 * r + g8 + 8 * (e >> 1), j = 16 * c + 8 * nt + 2 * tig + (e & 1);
                    T[i][j] = -Y[nt][e];
                }
            }
        };
        if (warp < 2) {
            const int r = warp ? 3 : 1, c = r - 1;
            float (*xb)[kLdF] = above(c, r);
            float X[2][4] = {}, Y[2][4] = {};
            mma_block16(X, L, 16 * r, 16 * c, T, 16 * c, 16 * c, g8, tig);
            store_block16(X, xb, g8, tig);
            __syncwarp();
            mma_block16(Y, T, 16 * r, 16 * r, xb, 0, 0, g8, tig);
            finish(r, c, Y);
        }
        __syncthreads();
        if (warp < 4) {
            const int i = 2 + (warp >> 1), j = warp & 1;
            // X_mj = sum over m' = j..1 of L_{m m'} T_{m' j}, for m = 2 (and m = 3 in row 3)
            float (*x2)[kLdF] = warp == 0 ? above(0, 1) : warp == 1 ? above(0, 2) : warp == 2 ? above(0, 3) : above(1, 3);
            float (*x3)[kLdF] = warp == 2 ? above(1, 2) : above(2, 3);
            float X[2][4] = {}, Y[2][4] = {};
            for (int m = j; m < 2; ++m) mma_block16(X, L, 32, 16 * m, T, 16 * m, 16 * j, g8, tig);
            store_block16(X, x2, g8, tig);
            if (i == 3) {
                float X3[2][4] = {};
                for (int m = j; m < 2; ++m) mma_block16(X3, L, 48, 16 * m, T, 16 * m, 16 * j, g8, tig);
                store_block16(X3, x3, g8, tig);
            }
            __syncwarp();
            if (i == 2) {
                mma_block16(Y, T, 32, 32, x2, 0, 0, g8, tig);  // T22 X_2j
            } else {
                mma_block16(Y, T, 48, 32, x2, 0, 0, g8, tig);  // T32 X_2j
                mma_block16(Y, T, 48, 48, x3, 0, 0, g8, tig);  // + T33 X_3j
            }
            finish(i, j, Y);
        }
        __syncthreads();
    }

    // Tw and Tu, eight columns per store (blocks above the diagonal are zero)
    for (int idx = tid; idx < PC * 8; idx += 256) {
        const int i = idx >> 3, j0 = 8 * (idx & 7);
        uint4 w = make_uint4(0u, 0u, 0u, 0u), u = w;
        if ((j0 >> 4) <= (i >> 4)) {
            const float4 t0 = *reinterpret_cast<const float4 *>(&s.t[i][j0]), t1 = *reinterpret_cast<const float4 *>(&s.t[i][j0 + 4]);
            const float4 f0 = *reinterpret_cast<const float4 *>(&s.fw[j0]), f1 = *reinterpret_cast<const float4 *>(&s.fw[j0 + 4]);
            const float4 b0 = *reinterpret_cast<const float4 *>(&s.beta[j0]), b1 = *reinterpret_cast<const float4 *>(&s.beta[j0 + 4]);
            w = make_uint4(pack_bf16(t0.x * f0.x, t0.y * f0.y), pack_bf16(t0.z * f0.z, t0.w * f0.w),
                           pack_bf16(t1.x * f1.x, t1.y * f1.y), pack_bf16(t1.z * f1.z, t1.w * f1.w));
            u = make_uint4(pack_bf16(t0.x * b0.x, t0.y * b0.y), pack_bf16(t0.z * b0.z, t0.w * b0.w),
                           pack_bf16(t1.x * b1.x, t1.y * b1.y), pack_bf16(t1.z * b1.z, t1.w * b1.w));
        }
        *reinterpret_cast<uint4 *>(tw + sw128(i, j0, PC)) = w;
        *reinterpret_cast<uint4 *>(tu + sw128(i, j0, PC)) = u;
    }

    // ---- raw v into the space of L (T is complete) while -W^T = K^T Tw^T runs
    {
        const bf16 *vg = static_cast<const bf16 *>(a.v);
        for (int idx = tid; idx < PC * 16; idx += 256) {
            const int row = idx >> 4, piece = idx & 15;
            unsigned char *dst = s.lv.v + sw128_mn(row, 8 * piece, PC);
            if (row < n) cp16(dst, vg + (int64_t(t0) + row) * a.v_stride + int64_t(head) * PV + piece * 8);
            else *reinterpret_cast<uint4 *>(dst) = make_uint4(0u, 0u, 0u, 0u);
        }
        asm volatile("cp.async.commit_group;\n" ::: "memory");
    }
    proxy_fence();  // Tw and Tu (generic stores) before the MMAs read them
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const bool run = !s.abort_flag;
    float g_next = 0.f, b_next = 0.f;  // the next head's gates, loaded while W and U are formed
    if (hr + 1 < R && tid < n) {
        const int64_t gi = (int64_t(t0) + tid) * H + head + 1;
        g_next = a.g[gi];
        b_next = a.beta[gi];
    }
    const uint32_t id_t = idesc_bf16_ab(PC, 1, 0);  // A MN-major (k or v as [token][key]), B K-major (Tw, Tu)
    // W^T, then U^T, in columns [64, 128): [K; Q] K^T stays in [0, 64) for the next head.
    if (run && tid == kIssuer) {
        const uint32_t qk = smem_addr(s.qk), b = smem_addr(tw);
#pragma unroll
        for (int ks = 0; ks < PC / 16; ++ks)
            umma(tmem + 64, sdesc(qk + ks * 2048, 16384, 1024), sdesc(b + ks * 32, 16, 1024), id_t, ks > 0);
        umma_commit(&s.bar);
    }
    asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    proxy_fence();
    if (run && !bar_wait(&s.bar, phase & 1)) s.abort_flag = 1;
    ++phase;
    tc_fence_after();
    const int r = 32 * (warp & 3) + lane, c0 = 32 * cq;  // r: key (W) and value (U); columns: tokens
    if (run) {  // -W (bf16, K-major tile) into the record
#pragma unroll 1
        for (int h = 0; h < 32; h += 16) {
            float x[16];
            tmem_ld16(tmem + tlane + 64 + c0 + h, x);
#pragma unroll
            for (int e = 0; e < 16; ++e)
                *reinterpret_cast<bf16 *>(rec + kRecW + sw128(c0 + h + e, r, PC)) = __float2bfloat16_rn(-x[e]);
        }
    }
    tc_fence_before();
    __syncthreads();  // W^T is read out; v (cp.async) is visible
    tc_fence_after();
    if (run && tid == kIssuer) {
        const uint32_t v = smem_addr(s.lv.v), b = smem_addr(tu);
#pragma unroll
        for (int ks = 0; ks < PC / 16; ++ks)
            umma(tmem + 64, sdesc(v + ks * 2048, 8192, 1024), sdesc(b + ks * 32, 16, 1024), id_t, ks > 0);
        umma_commit(&s.bar);
    }
    if (run && !bar_wait(&s.bar, phase & 1)) s.abort_flag = 1;
    ++phase;
    tc_fence_after();
    if (run) {  // U (bf16 row-major) into the record
        bf16 *urec = reinterpret_cast<bf16 *>(rec + kRecU);
#pragma unroll 1
        for (int h = 0; h < 32; h += 16) {
            float x[16];
            tmem_ld16(tmem + tlane + 64 + c0 + h, x);
#pragma unroll
            for (int e = 0; e < 16; ++e) urec[(c0 + h + e) * PV + r] = __float2bfloat16_rn(x[e]);
        }
    }
    if (tid < PC) {
        const float gC = s.gam[PC - 1];
        reinterpret_cast<float *>(rec + kRecRo)[tid] = expf(s.gam[tid]) * s.nq[tid] * a.scale;
        reinterpret_cast<float *>(rec + kRecRd)[tid] = expf(gC - s.gam[tid]) * s.nk[tid];
        if (tid == 0) reinterpret_cast<float *>(rec + kRecDc)[0] = expf(gC);
    }
    tc_fence_before();
    __syncthreads();  // every read of this head's gates, L, T and tiles is done
    tc_fence_after();
    if (hr + 1 < R && tid < PC) {
        s.gam[tid] = g_next;
        s.beta[tid] = b_next;
    }
    __syncthreads();
    }  // value heads of the group
    if (s.abort_flag && tid == 0 && a.status) atomicOr(a.status, SQ_STATUS_TIMEOUT);
    tc_fence_before();
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" :: "r"(tmem), "r"(kPrepCols));
}

__global__ void __launch_bounds__(512, 1) state_kernel(sq_prefill_args a, const int32_t *offsets,
                                                       const unsigned char *records) {
    extern __shared__ unsigned char smem_raw[];
    // 1024-byte aligned (swizzle atoms); offsetting the shared array keeps its address space.
    TcSmem &s = *reinterpret_cast<TcSmem *>(smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u));
    __shared__ uint64_t bar_data[2], bar_mma[2];
    __shared__ uint32_t tmem_slot;
    __shared__ int abort_flag;
    const int tid = threadIdx.x, warp = tid >> 5;
    const int H = a.heads;
    const int seq = blockIdx.x / H, head = blockIdx.x % H;
    const int qh = head / (H / a.qk_heads);
    const int2 range = seq_range(a, seq);
    const int chunks = (range.y - range.x + PC - 1) / PC;
    const unsigned char *rec0 = records + (int64_t(offsets[seq]) * H + head) * kRec;
    bf16 *og = static_cast<bf16 *>(a.out);
    const int v = 32 * (warp & 3) + (tid & 31);  // value column = TMEM lane
    const int cq = warp >> 2;                     // column quarter of every accumulator

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" :: "r"(smem_addr(&tmem_slot)), "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n");
    }
    if (tid == 0) {
        for (int i = 0; i < 2; ++i) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" :: "r"(smem_addr(&bar_data[i])));
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" :: "r"(smem_addr(&bar_mma[i])));
        }
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        abort_flag = 0;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    const uint32_t lane = uint32_t(32 * (warp & 3)) << 16;

    // Initial state: S^T row v = column v of S.
    {
        const float *init = a.initial_state ? a.initial_state + (int64_t(seq) * H + head) * PK * PV : nullptr;
        const int k0 = 32 * cq;
        float x[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) x[j] = init ? init[(k0 + j) * PV + v] : 0.f;
        tmem_st32(tmem + lane + kColS + k0, x);
        put_row<32>(s.sb, PK, v, k0, x);
        asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
    }
    // Chunk c uses D and O1 columns of parity c & 1, so the next chunk's first
    // MMAs (into the other pair) run while chunk c's outputs are read out.
    auto col_d = [](int parity) { return parity ? kColD1 : kColD; };
    auto col_o1 = [](int parity) { return parity ? kColO11 : kColO1; };
    const uint32_t id64 = idesc_bf16(64, 0), id128mn = idesc_bf16(128, 1);
    auto issue_first = [&](const TcStage &st, int parity) {  // D^T = S^T (-W)^T, O1^T = S^T Q^T
        const uint32_t sb = smem_addr(s.sb), w = smem_addr(st.w), q = smem_addr(st.q);
#pragma unroll
        for (int ks = 0; ks < PK / 16; ++ks) {
            const uint32_t ao = (ks >> 2) * 16384 + (ks & 3) * 32, bo = (ks >> 2) * 8192 + (ks & 3) * 32;
            umma(tmem + col_d(parity), sdesc(sb + ao, 16, 1024), sdesc(w + bo, 16, 1024), id64, ks > 0);
            umma(tmem + col_o1(parity), sdesc(sb + ao, 16, 1024), sdesc(q + bo, 16, 1024), id64, ks > 0);
        }
        umma_commit(&bar_mma[0]);
    };
    if (chunks > 0) {
        tc_stage(a, s.st[0], &bar_data[0], rec0, range.x, min(PC, range.y - range.x), qh, tid);
        asm volatile("cp.async.commit_group;\n" ::: "memory");
        asm volatile("cp.async.wait_group 0;\n" ::: "memory");
        proxy_fence();
        if (!bar_wait(&bar_data[0], 0)) abort_flag = 1;
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        if (!abort_flag && tid == 0) issue_first(s.st[0], 0);
        if (chunks > 1)
            tc_stage(a, s.st[1], &bar_data[1], rec0 + int64_t(H) * kRec, range.x + PC, min(PC, range.y - range.x - PC),
                     qh, tid);
        asm volatile("cp.async.commit_group;\n" ::: "memory");
    }

    for (int c = 0; c < chunks; ++c) {
        if (abort_flag) break;
        const int par = c & 1;
        TcStage &st = s.st[par];
        const int t0 = range.x + c * PC, n = min(PC, range.y - t0);
        if (!bar_wait(&bar_mma[0], c & 1)) abort_flag = 1;
        tc_fence_after();

        // ---- D = U + D; D^T and Dt^T tiles; S^T *= e^gam_C
        {
            const bf16 *u = reinterpret_cast<const bf16 *>(st.u);
            const int tq = 16 * cq;
            float d[16], dt[16];
            tmem_ld16(tmem + lane + col_d(par) + tq, d);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                d[j] += __bfloat162float(u[(tq + j) * PV + v]);
                dt[j] = st.rd[tq + j] * d[j];
            }
            put_row<16>(s.dm, PK, v, tq, d);
            put_row<16>(s.dtm, PK, v, tq, dt);
            const float dc = st.dc[0];
            float x[32];
            tmem_ld32(tmem + lane + kColS + 32 * cq, x);
#pragma unroll
            for (int j = 0; j < 32; ++j) x[j] *= dc;
            tmem_st32(tmem + lane + kColS + 32 * cq, x);
            asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
        }
        proxy_fence();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        if (abort_flag) break;

        // ---- O2^T = D^T P^T, S^T += Dt^T K
        if (tid == 0) {
            const uint32_t dm = smem_addr(s.dm), dtm = smem_addr(s.dtm), pp = smem_addr(st.p), k = smem_addr(st.k);
#pragma unroll
            for (int ks = 0; ks < PC / 16; ++ks) {
                umma(tmem + kColO2, sdesc(dm + ks * 32, 16, 1024), sdesc(pp + ks * 32, 16, 1024), id64, ks > 0);
                umma(tmem + kColS, sdesc(dtm + ks * 32, 16, 1024), sdesc(k + ks * 2048, 8192, 1024), id128mn, 1);
            }
            umma_commit(&bar_mma[1]);
        }
        if (!bar_wait(&bar_mma[1], c & 1)) abort_flag = 1;
        tc_fence_after();

        // ---- the bf16 state tile for the next chunk; its copies; its first MMAs
        {
            float x[32];
            tmem_ld32(tmem + lane + kColS + 32 * cq, x);
            put_row<32>(s.sb, PK, v, 32 * cq, x);
        }
        if (c + 1 < chunks) {
            asm volatile("cp.async.wait_group 0;\n" ::: "memory");
            if (!bar_wait(&bar_data[par ^ 1], ((c + 1) >> 1) & 1)) abort_flag = 1;
        }
        proxy_fence();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        if (c + 1 < chunks && !abort_flag && tid == 0) issue_first(s.st[par ^ 1], par ^ 1);

        // ---- outputs o_t = ro_t (Q S)_t + (P D)_t, while the next chunk's MMAs run
        {
            const int tq = 16 * cq;
            float o1[16], o2[16];
            tmem_ld16(tmem + lane + col_o1(par) + tq, o1);
            tmem_ld16(tmem + lane + kColO2 + tq, o2);
            bf16 *orow = og + ((int64_t(t0) + tq) * H + head) * PV + v;
            const int64_t ostride = int64_t(H) * PV;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                if (tq + j < n) orow[j * ostride] = __float2bfloat16_rn(st.ro[tq + j] * o1[j] + o2[j]);
            }
        }
        // Every read of this stage buffer is done: refill it with chunk c + 2.
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        if (c + 2 < chunks)
            tc_stage(a, st, &bar_data[par], rec0 + int64_t(c + 2) * H * kRec, t0 + 2 * PC,
                     min(PC, range.y - t0 - 2 * PC), qh, tid);
        asm volatile("cp.async.commit_group;\n" ::: "memory");
    }
    asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (abort_flag) {
        if (tid == 0 && a.status) atomicOr(a.status, SQ_STATUS_TIMEOUT);
    } else {
        float *fin = a.final_state + (int64_t(seq) * H + head) * PK * PV;
        float x[32];
        tmem_ld32(tmem + lane + kColS + 32 * cq, x);
#pragma unroll
        for (int j = 0; j < 32; ++j) fin[(32 * cq + j) * PV + v] = x[j];
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" :: "r"(tmem), "r"(kTmemCols));
}

bool aligned_rows(const void *p, int64_t stride) {
    return (reinterpret_cast<uintptr_t>(p) & 15u) == 0 && (stride * 2) % 16 == 0;
}

int64_t max_chunks(int64_t tokens, int64_t seqs) { return (tokens + PC - 1) / PC + seqs; }

}  // namespace
}  // namespace sq

extern "C" int64_t sq_gdn_prefill_workspace_bytes(int32_t tokens, int32_t num_seqs, int32_t heads) {
    if (tokens < 0 || num_seqs < 0 || heads < 1) return -1;
    const int64_t chunks = sq::max_chunks(tokens, num_seqs);
    return sq::kOffsetsBytes(num_seqs) + sq::kChunkTabBytes(chunks) + chunks * heads * int64_t(sq::kRec);
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
    const int64_t chunks = sq::max_chunks(a.tokens, a.num_seqs);
    if (chunks > 0x7fffffff) return SQ_ERR_SHAPE;
    int2 *chunk_tab = reinterpret_cast<int2 *>(static_cast<unsigned char *>(a.workspace) + sq::kOffsetsBytes(a.num_seqs));
    unsigned char *records = reinterpret_cast<unsigned char *>(chunk_tab) + sq::kChunkTabBytes(chunks);
    sq::offsets_kernel<<<1, 1024, 0, s>>>(a, offsets, chunk_tab);
    const int prep_smem = sq::kPrepSmemBytes, state_smem = int(sizeof(sq::TcSmem)) + 1024;
    if (cudaFuncSetAttribute(sq::prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, prep_smem) != cudaSuccess ||
        cudaFuncSetAttribute(sq::state_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, state_smem) != cudaSuccess)
        return SQ_ERR_CUDA;
    if (chunks * a.qk_heads > 0x7fffffff) return SQ_ERR_SHAPE;
    if (chunks > 0) sq::prep_kernel<<<unsigned(chunks * a.qk_heads), 256, prep_smem, s>>>(a, offsets, chunk_tab, records);
    sq::state_kernel<<<a.num_seqs * a.heads, 512, state_smem, s>>>(a, offsets, records);
    return cudaGetLastError() == cudaSuccess ? SQ_OK : SQ_ERR_CUDA;
}
