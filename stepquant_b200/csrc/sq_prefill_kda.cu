// KDA prefill: the state pass that produces each sequence's state after its
// prompt for layers with a per-key-channel decay.  In the reference it is
// SGLang's KDA chunk kernel, called by the prefill hook between
// PackedStatePool.decode and PackedStatePool.encode
// (stepquant/sglang/runtime.py:193-202); the recurrence it evaluates is
// core.delta_step (stepquant/core.py:5-15) token by token with log_decay of
// shape [H, K]:
//     S <- diag(e^g) S;  d = beta (v - S^T k);  S <- S + k d^T;  o = S^T q.
//
// One 256-thread CTA per (sequence, value head), two per SM, the fp32 state
// in registers for the whole prompt (read once, written once).  Lane l of
// warp w holds rows 16 (l % 8) .. 16 (l % 8) + 15 of the four columns
// 16 w + 4 (l / 8) .. + 3: the eight lanes of a quarter-warp share a column
// group and cover all 128 rows.  Per token a lane reads its 16 rows of e^g, k
// and q (twelve 16-byte shared loads; the 16-row chunks are 20 floats apart,
// so the eight chunks a quarter-warp reads fill the 32 banks once), forms the
// 8 partial column sums (k and q for 4 columns) over its rows, and the
// column group reduces them by recursive halving (7 shuffles, each lane ends
// with one total), the k lanes form d = beta (v - S^T k), the q lanes
// o = S^T q + (q . k) d, and d reaches every lane of the group (4 shuffles)
// for the rank-1 update.
// Tokens are staged in blocks of 16: the next block's q, k, v and g rows
// arrive by cp.async while the current block runs, and a prologue per block
// normalises q and k and forms e^g, beta and q . k in shared memory.
// Arithmetic is fp32 (products in packed f32x2 form over row pairs), so the
// result matches the fp32 recurrence up to rounding order.
#include <cuda_runtime.h>

#include "sq_fast.cuh"

namespace sq {
namespace {

constexpr int KK = 128;           // keys
constexpr int KV = 128;           // values
constexpr int KTB = 16;           // tokens per staged block
constexpr int kKpThreads = 256;
constexpr int kPieces = 16 + 16 + 16 + 32;  // 16-byte pieces of one token: q, k, v (bf16), g (fp32)
constexpr int kChunk = 20;                  // floats per 16-key chunk of a prepared row (16 + 4 pad)
constexpr int kRowPad = 8 * kChunk;
__device__ __forceinline__ int kq_at(int key) { return (key >> 4) * kChunk + (key & 15); }

struct KdaPrefillRaw {
    __nv_bfloat16 q[KTB][KK];
    __nv_bfloat16 k[KTB][KK];
    __nv_bfloat16 v[KTB][KV];
    float g[KTB][KK];
};

struct KdaPrefillSmem {
    KdaPrefillRaw raw[2];
    float qn[KTB][kRowPad];  // q / |q| * scale   (key i at kq_at(i))
    float kn[KTB][kRowPad];  // k / |k|
    float e[KTB][kRowPad];   // e^g
    float beta[KTB];
    float qk[KTB];           // (q / |q| * scale) . (k / |k|)
};

__device__ __forceinline__ int2 kda_seq_range(const sq_prefill_args &a, int n) {
    const int b = max(0, min(a.cu_seqlens[n], a.tokens));
    return make_int2(b, max(b, min(a.cu_seqlens[n + 1], a.tokens)));
}

// cp.async of tokens t0 .. t0 + n - 1 (row bases are 16-byte aligned: checked
// by the entry point).
__device__ __forceinline__ void kda_stage(KdaPrefillRaw &r, const sq_prefill_args &a, int t0, int n, int head, int qh,
                                          int tid) {
    for (int i = tid; i < n * kPieces; i += kKpThreads) {
        const int j = i / kPieces, p = i - j * kPieces;
        const int64_t t = t0 + j;
        const unsigned char *src;
        unsigned char *dst;
        if (p < 16) {
            src = static_cast<const unsigned char *>(a.q) + 2 * (t * a.q_stride + int64_t(qh) * KK) + 16 * p;
            dst = reinterpret_cast<unsigned char *>(r.q[j]) + 16 * p;
        } else if (p < 32) {
            src = static_cast<const unsigned char *>(a.k) + 2 * (t * a.k_stride + int64_t(qh) * KK) + 16 * (p - 16);
            dst = reinterpret_cast<unsigned char *>(r.k[j]) + 16 * (p - 16);
        } else if (p < 48) {
            src = static_cast<const unsigned char *>(a.v) + 2 * (t * a.v_stride + int64_t(head) * KV) + 16 * (p - 32);
            dst = reinterpret_cast<unsigned char *>(r.v[j]) + 16 * (p - 32);
        } else {
            src = reinterpret_cast<const unsigned char *>(a.g + (t * a.heads + head) * KK) + 16 * (p - 48);
            dst = reinterpret_cast<unsigned char *>(r.g[j]) + 16 * (p - 48);
        }
        cp_async16(dst, src);
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
}

// Per-block prologue: thread (j, part) = (tid / 16, tid % 16) covers keys
// 8 part .. 8 part + 7 of token j (one prepared chunk); the squared norms and
// q . k are summed over the token's 16 lanes by shuffles.
__device__ __forceinline__ void kda_prepare(KdaPrefillSmem &s, const KdaPrefillRaw &r, const sq_prefill_args &a,
                                            int t0, int n, int head, int tid) {
    const int j = tid >> 4, part = tid & 15;
    const bool on = j < n;
    float q[8], k[8];
    if (on) {
        const uint4 qb = *reinterpret_cast<const uint4 *>(&r.q[j][8 * part]);
        const uint4 kb = *reinterpret_cast<const uint4 *>(&r.k[j][8 * part]);
        const uint32_t qw[4] = {qb.x, qb.y, qb.z, qb.w}, kw[4] = {kb.x, kb.y, kb.z, kb.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 qf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&qw[i]));
            const float2 kf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&kw[i]));
            q[2 * i] = qf.x;
            q[2 * i + 1] = qf.y;
            k[2 * i] = kf.x;
            k[2 * i + 1] = kf.y;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = k[i] = 0.f;
    }
    float qq = 0.f, kk = 0.f, qk = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        qq = fmaf(q[i], q[i], qq);
        kk = fmaf(k[i], k[i], kk);
        qk = fmaf(q[i], k[i], qk);
    }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) {  // within the token's 16 lanes
        qq += __shfl_xor_sync(0xffffffffu, qq, o);
        kk += __shfl_xor_sync(0xffffffffu, kk, o);
        qk += __shfl_xor_sync(0xffffffffu, qk, o);
    }
    if (!on) return;
    const float qs = (a.normalize ? __frsqrt_rn(qq + 1e-6f) : 1.f) * a.scale;
    const float ks = a.normalize ? __frsqrt_rn(kk + 1e-6f) : 1.f;
    const float4 g0 = *reinterpret_cast<const float4 *>(&r.g[j][8 * part]);
    const float4 g1 = *reinterpret_cast<const float4 *>(&r.g[j][8 * part + 4]);
    float4 *qd = reinterpret_cast<float4 *>(&s.qn[j][kq_at(8 * part)]);
    float4 *kd = reinterpret_cast<float4 *>(&s.kn[j][kq_at(8 * part)]);
    float4 *ed = reinterpret_cast<float4 *>(&s.e[j][kq_at(8 * part)]);
    qd[0] = make_float4(q[0] * qs, q[1] * qs, q[2] * qs, q[3] * qs);
    qd[1] = make_float4(q[4] * qs, q[5] * qs, q[6] * qs, q[7] * qs);
    kd[0] = make_float4(k[0] * ks, k[1] * ks, k[2] * ks, k[3] * ks);
    kd[1] = make_float4(k[4] * ks, k[5] * ks, k[6] * ks, k[7] * ks);
    ed[0] = make_float4(expf(g0.x), expf(g0.y), expf(g0.z), expf(g0.w));
    ed[1] = make_float4(expf(g1.x), expf(g1.y), expf(g1.z), expf(g1.w));
    if (part == 0) {
        s.beta[j] = a.beta[int64_t(t0 + j) * a.heads + head];
        s.qk[j] = qk * qs * ks;
    }
}

__device__ __forceinline__ float2 lo_pair(float4 v) { return make_float2(v.x, v.y); }
__device__ __forceinline__ float2 hi_pair(float4 v) { return make_float2(v.z, v.w); }

// Tokens of one staged block.  S[p][c]: rows 16 (lane % 8) + 2 p and + 1 of
// column col0 + c, col0 = 16 warp + 4 (lane / 8).
__device__ __forceinline__ void kda_block(const KdaPrefillSmem &s, const KdaPrefillRaw &r, const sq_prefill_args &a,
                                          int t0, int n, int head, int lane, int col0, float2 (&S)[8][4]) {
    __nv_bfloat16 *out = static_cast<__nv_bfloat16 *>(a.out);
    const int c8 = lane & 7, src0 = lane & 24;
    const int col = col0 + (c8 >> 1);  // the column of this lane's total
    const bool is_q = (c8 & 1) != 0;   // totals: k sums on even lanes, q sums on odd lanes
#pragma unroll 1
    for (int j = 0; j < n; ++j) {
        const float4 *e4 = reinterpret_cast<const float4 *>(&s.e[j][kChunk * c8]);
        const float4 *k4 = reinterpret_cast<const float4 *>(&s.kn[j][kChunk * c8]);
        const float4 *q4 = reinterpret_cast<const float4 *>(&s.qn[j][kChunk * c8]);
        float2 K[8];
#pragma unroll
        for (int h = 0; h < 4; ++h) {
            const float4 kv = k4[h];
            K[2 * h] = lo_pair(kv);
            K[2 * h + 1] = hi_pair(kv);
        }
        float sums[8];  // 2 c: the lane's part of (S^T k)_c, 2 c + 1: of (S^T q)_c, after the decay
        {
            float2 ak[4], aq[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) ak[c] = aq[c] = make_float2(0.f, 0.f);
#pragma unroll
            for (int h = 0; h < 4; ++h) {
                const float4 ev = e4[h], qv = q4[h];
                const float2 E0 = lo_pair(ev), E1 = hi_pair(ev), Q0 = lo_pair(qv), Q1 = hi_pair(qv);
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    S[2 * h][c] = pmul2(S[2 * h][c], E0);
                    S[2 * h + 1][c] = pmul2(S[2 * h + 1][c], E1);
                    ak[c] = pfma2(K[2 * h], S[2 * h][c], ak[c]);
                    aq[c] = pfma2(Q0, S[2 * h][c], aq[c]);
                    ak[c] = pfma2(K[2 * h + 1], S[2 * h + 1][c], ak[c]);
                    aq[c] = pfma2(Q1, S[2 * h + 1][c], aq[c]);
                }
            }
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                sums[2 * c] = ak[c].x + ak[c].y;
                sums[2 * c + 1] = aq[c].x + aq[c].y;
            }
        }
        // Recursive halving over the 8 lanes of the column group: at mask m a
        // lane keeps the upper half of its values when (lane & m), adds the
        // partner's copy of that half and passes on the other; lane c8 ends
        // with total c8.
        float h4[4], h2[2];
        {
            const bool up = (c8 & 4) != 0;
#pragma unroll
            for (int i = 0; i < 4; ++i)
                h4[i] = (up ? sums[i + 4] : sums[i]) + __shfl_xor_sync(0xffffffffu, up ? sums[i] : sums[i + 4], 4);
        }
        {
            const bool up = (c8 & 2) != 0;
#pragma unroll
            for (int i = 0; i < 2; ++i)
                h2[i] = (up ? h4[i + 2] : h4[i]) + __shfl_xor_sync(0xffffffffu, up ? h4[i] : h4[i + 2], 2);
        }
        const float total = (is_q ? h2[1] : h2[0]) + __shfl_xor_sync(0xffffffffu, is_q ? h2[0] : h2[1], 1);
        // k lanes: d = beta (v - S^T k); q lanes take it from their k lane and store o.
        float d = s.beta[j] * (__bfloat162float(r.v[j][col]) - total);
        const float dk = __shfl_xor_sync(0xffffffffu, d, 1);
        if (is_q) {
            d = dk;
            out[(int64_t(t0 + j) * a.heads + head) * KV + col] = __float2bfloat16_rn(total + s.qk[j] * d);
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const float dc = __shfl_sync(0xffffffffu, d, src0 + 2 * c);
            const float2 dd = make_float2(dc, dc);
#pragma unroll
            for (int p = 0; p < 8; ++p) S[p][c] = pfma2(K[p], dd, S[p][c]);
        }
    }
}

__global__ void __launch_bounds__(kKpThreads, 2) kda_prefill_kernel(sq_prefill_args a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    KdaPrefillSmem &s = *reinterpret_cast<KdaPrefillSmem *>(smem_raw);
    const int seq = blockIdx.x / a.heads, head = blockIdx.x - seq * a.heads;
    const int qh = head / (a.heads / a.qk_heads);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int row0 = 16 * (lane & 7), col0 = 16 * warp + 4 * (lane >> 3);
    const int2 range = kda_seq_range(a, seq);
    const int64_t base = (int64_t(seq) * a.heads + head) * KK * KV;
    const int blocks = (range.y - range.x + KTB - 1) / KTB;
    if (blocks > 0) kda_stage(s.raw[0], a, range.x, min(KTB, range.y - range.x), head, qh, tid);

    float2 S[8][4];
    if (a.initial_state) {
        const float *init = a.initial_state + base;
#pragma unroll
        for (int p = 0; p < 8; ++p) {
            const float4 r0 = *reinterpret_cast<const float4 *>(init + (row0 + 2 * p) * KV + col0);
            const float4 r1 = *reinterpret_cast<const float4 *>(init + (row0 + 2 * p + 1) * KV + col0);
            S[p][0] = make_float2(r0.x, r1.x);
            S[p][1] = make_float2(r0.y, r1.y);
            S[p][2] = make_float2(r0.z, r1.z);
            S[p][3] = make_float2(r0.w, r1.w);
        }
    } else {
#pragma unroll
        for (int p = 0; p < 8; ++p)
#pragma unroll
            for (int c = 0; c < 4; ++c) S[p][c] = make_float2(0.f, 0.f);
    }

#pragma unroll 1
    for (int b = 0; b < blocks; ++b) {
        const int t0 = range.x + b * KTB, n = min(KTB, range.y - t0);
        if (b + 1 < blocks) {  // the next block's copies run beside this block
            kda_stage(s.raw[(b + 1) & 1], a, t0 + KTB, min(KTB, range.y - t0 - KTB), head, qh, tid);
            asm volatile("cp.async.wait_group 1;\n" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;\n" ::: "memory");
        }
        __syncthreads();  // block b staged for every thread
        kda_prepare(s, s.raw[b & 1], a, t0, n, head, tid);
        __syncthreads();
        kda_block(s, s.raw[b & 1], a, t0, n, head, lane, col0, S);
        __syncthreads();  // prepared rows and raw[b & 1] are free again
    }

    float *fin = a.final_state + base;
#pragma unroll
    for (int p = 0; p < 8; ++p) {
        *reinterpret_cast<float4 *>(fin + (row0 + 2 * p) * KV + col0) = make_float4(S[p][0].x, S[p][1].x, S[p][2].x, S[p][3].x);
        *reinterpret_cast<float4 *>(fin + (row0 + 2 * p + 1) * KV + col0) =
            make_float4(S[p][0].y, S[p][1].y, S[p][2].y, S[p][3].y);
    }
}

bool kda_aligned_rows(const void *p, int64_t stride) {
    return (reinterpret_cast<uintptr_t>(p) & 15u) == 0 && (stride * 2) % 16 == 0;
}

}  // namespace
}  // namespace sq

extern "C" int32_t sq_kda_prefill(const sq_prefill_args *args, sq_stream_t stream) {
    if (!args) return SQ_ERR_ARGUMENT;
    const sq_prefill_args &a = *args;
    if (a.num_seqs < 0 || a.tokens < 0 || a.heads < 1 || a.qk_heads < 1) return SQ_ERR_ARGUMENT;
    if (a.heads % a.qk_heads) return SQ_ERR_SHAPE;
    if (a.keys != sq::KK || a.values != sq::KV || a.io_dtype != SQ_BF16) return SQ_ERR_UNSUPPORTED;
    if (a.num_seqs == 0) return SQ_OK;
    if (!a.q || !a.k || !a.v || !a.g || !a.beta || !a.cu_seqlens || !a.final_state || !a.out) return SQ_ERR_ARGUMENT;
    if (a.q_stride < 0 || a.k_stride < 0 || a.v_stride < 0) return SQ_ERR_SHAPE;
    if (!sq::kda_aligned_rows(a.q, a.q_stride) || !sq::kda_aligned_rows(a.k, a.k_stride) ||
        !sq::kda_aligned_rows(a.v, a.v_stride) || (reinterpret_cast<uintptr_t>(a.g) & 15u) ||
        (reinterpret_cast<uintptr_t>(a.out) & 1u) || (reinterpret_cast<uintptr_t>(a.final_state) & 15u) ||
        (reinterpret_cast<uintptr_t>(a.initial_state) & 15u))
        return SQ_ERR_SHAPE;
    if (int64_t(a.num_seqs) * a.heads > 0x7fffffff) return SQ_ERR_SHAPE;
    const int smem = int(sizeof(sq::KdaPrefillSmem));
    if (cudaFuncSetAttribute(sq::kda_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
        return SQ_ERR_CUDA;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    sq::kda_prefill_kernel<<<unsigned(int64_t(a.num_seqs) * a.heads), sq::kKpThreads, smem, s>>>(a);
    return cudaGetLastError() == cudaSuccess ? SQ_OK : SQ_ERR_CUDA;
}
