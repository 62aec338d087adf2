// KDA prefill: the state pass that produces each sequence's state after its
// prompt for layers with a per-key-channel decay.  In the reference it is
// SGLang's KDA chunk kernel, called by the prefill hook between
// PackedStatePool.decode and PackedStatePool.encode
// (stepquant/sglang/runtime.py:193-202); the recurrence it evaluates is
// core.delta_step (stepquant/core.py:5-15) token by token with log_decay of
// shape [H, K]:
//     S <- diag(e^g) S;  d = beta (v - S^T k);  S <- S + k d^T;  o = S^T q.
//
// One 256-thread CTA per (sequence, value head), two per SM.  Thread t keeps
// columns c and c + 64 (c = t / 4) of the fp32 state, rows 32 (t % 4) ..
// 32 (t % 4) + 31, in registers for the whole prompt: the state is read once
// and written once, and the per-token column sums S^T k and S^T q are the
// thread's 32-row partials plus those of the three other lanes of its
// quad (two shuffles each, no barrier).  o = S_dec^T q + (q . k) d, with
// S_dec the decayed state, so one pass over the state forms both sums.
// Tokens are taken in blocks of 16: the next block's q, k, v and g rows are
// staged by cp.async while the current block runs, and a short prologue per
// block normalises q and k, forms e^g, beta and q . k in shared memory.
// Arithmetic is fp32 (products in packed f32x2 form), so the result matches
// the fp32 recurrence up to summation order.
#include <cuda_runtime.h>

#include "sq_fast.cuh"

namespace sq {
namespace {

constexpr int KK = 128;           // keys
constexpr int KV = 128;           // values
constexpr int KTB = 16;           // tokens per staged block
constexpr int kKpThreads = 256;
constexpr int kPieces = 16 + 16 + 16 + 32;  // 16-byte pieces of one token: q, k, v (bf16), g (fp32)
// Prepared rows keep the four 32-key quarters 36 floats apart, so that the
// four lanes of a quad (one quarter each) read distinct banks.
constexpr int kRowPad = 4 * 36;
__device__ __forceinline__ int kq_at(int key) { return (key >> 5) * 36 + (key & 31); }

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
    float qk[KTB];      // (q / |q| * scale) . (k / |k|)
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

// Per-block prologue: thread (j, part) = (tid / 16, tid % 16) covers elements
// 8 part .. 8 part + 7 of token j; the squared norms and q . k are summed over
// the token's 16 lanes by shuffles.
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

// Tokens of one staged block.  S0 / S1: columns c / c + 64, element i holding
// rows 32 qd + 2 i and 32 qd + 2 i + 1.
__device__ __forceinline__ void kda_block(const KdaPrefillSmem &s, const KdaPrefillRaw &r, const sq_prefill_args &a,
                                          int t0, int n, int head, int qd, int c, float2 (&S0)[16], float2 (&S1)[16]) {
    __nv_bfloat16 *out = static_cast<__nv_bfloat16 *>(a.out);
#pragma unroll 1
    for (int j = 0; j < n; ++j) {
        const float4 *e4 = reinterpret_cast<const float4 *>(&s.e[j][36 * qd]);
        const float4 *k4 = reinterpret_cast<const float4 *>(&s.kn[j][36 * qd]);
        const float4 *q4 = reinterpret_cast<const float4 *>(&s.qn[j][36 * qd]);
        float2 ak0 = make_float2(0.f, 0.f), aq0 = ak0, ak1 = ak0, aq1 = ak0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 ev = e4[i], kv = k4[i], qv = q4[i];
            S0[2 * i] = pmul2(S0[2 * i], lo_pair(ev));
            S0[2 * i + 1] = pmul2(S0[2 * i + 1], hi_pair(ev));
            S1[2 * i] = pmul2(S1[2 * i], lo_pair(ev));
            S1[2 * i + 1] = pmul2(S1[2 * i + 1], hi_pair(ev));
            ak0 = pfma2(lo_pair(kv), S0[2 * i], ak0);
            ak0 = pfma2(hi_pair(kv), S0[2 * i + 1], ak0);
            aq0 = pfma2(lo_pair(qv), S0[2 * i], aq0);
            aq0 = pfma2(hi_pair(qv), S0[2 * i + 1], aq0);
            ak1 = pfma2(lo_pair(kv), S1[2 * i], ak1);
            ak1 = pfma2(hi_pair(kv), S1[2 * i + 1], ak1);
            aq1 = pfma2(lo_pair(qv), S1[2 * i], aq1);
            aq1 = pfma2(hi_pair(qv), S1[2 * i + 1], aq1);
        }
        float ks0 = ak0.x + ak0.y, qs0 = aq0.x + aq0.y, ks1 = ak1.x + ak1.y, qs1 = aq1.x + aq1.y;
#pragma unroll
        for (int o = 1; o < 4; o <<= 1) {  // the quad's four row ranges
            ks0 += __shfl_xor_sync(0xffffffffu, ks0, o);
            qs0 += __shfl_xor_sync(0xffffffffu, qs0, o);
            ks1 += __shfl_xor_sync(0xffffffffu, ks1, o);
            qs1 += __shfl_xor_sync(0xffffffffu, qs1, o);
        }
        const float b = s.beta[j], qk = s.qk[j];
        const float d0 = b * (__bfloat162float(r.v[j][c]) - ks0);
        const float d1 = b * (__bfloat162float(r.v[j][c + 64]) - ks1);
        const float2 dd0 = make_float2(d0, d0), dd1 = make_float2(d1, d1);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 kv = k4[i];
            S0[2 * i] = pfma2(lo_pair(kv), dd0, S0[2 * i]);
            S0[2 * i + 1] = pfma2(hi_pair(kv), dd0, S0[2 * i + 1]);
            S1[2 * i] = pfma2(lo_pair(kv), dd1, S1[2 * i]);
            S1[2 * i + 1] = pfma2(hi_pair(kv), dd1, S1[2 * i + 1]);
        }
        const int64_t row = (int64_t(t0 + j) * a.heads + head) * KV;
        if (qd == 0) out[row + c] = __float2bfloat16_rn(qs0 + qk * d0);
        if (qd == 1) out[row + c + 64] = __float2bfloat16_rn(qs1 + qk * d1);
    }
}

__global__ void __launch_bounds__(kKpThreads, 2) kda_prefill_kernel(sq_prefill_args a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    KdaPrefillSmem &s = *reinterpret_cast<KdaPrefillSmem *>(smem_raw);
    const int seq = blockIdx.x / a.heads, head = blockIdx.x - seq * a.heads;
    const int qh = head / (a.heads / a.qk_heads);
    const int tid = threadIdx.x, qd = tid & 3, c = tid >> 2;
    const int2 range = kda_seq_range(a, seq);
    const int64_t base = (int64_t(seq) * a.heads + head) * KK * KV;
    const int blocks = (range.y - range.x + KTB - 1) / KTB;
    if (blocks > 0) kda_stage(s.raw[0], a, range.x, min(KTB, range.y - range.x), head, qh, tid);

    float2 S0[16], S1[16];
    if (a.initial_state) {
        const float *init = a.initial_state + base;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int r = 32 * qd + 2 * i;
            S0[i] = make_float2(init[r * KV + c], init[(r + 1) * KV + c]);
            S1[i] = make_float2(init[r * KV + c + 64], init[(r + 1) * KV + c + 64]);
        }
    } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) S0[i] = S1[i] = make_float2(0.f, 0.f);
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
        kda_block(s, s.raw[b & 1], a, t0, n, head, qd, c, S0, S1);
        __syncthreads();  // prepared rows and raw[b & 1] are free again
    }

    float *fin = a.final_state + base;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const int r = 32 * qd + 2 * i;
        fin[r * KV + c] = S0[i].x;
        fin[(r + 1) * KV + c] = S0[i].y;
        fin[r * KV + c + 64] = S1[i].x;
        fin[(r + 1) * KV + c + 64] = S1[i].y;
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
        (reinterpret_cast<uintptr_t>(a.out) & 1u) || (reinterpret_cast<uintptr_t>(a.final_state) & 3u) ||
        (reinterpret_cast<uintptr_t>(a.initial_state) & 3u))
        return SQ_ERR_SHAPE;
    if (int64_t(a.num_seqs) * a.heads > 0x7fffffff) return SQ_ERR_SHAPE;
    const int smem = int(sizeof(sq::KdaPrefillSmem));
    if (cudaFuncSetAttribute(sq::kda_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
        return SQ_ERR_CUDA;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    sq::kda_prefill_kernel<<<unsigned(int64_t(a.num_seqs) * a.heads), sq::kKpThreads, smem, s>>>(a);
    return cudaGetLastError() == cudaSuccess ? SQ_OK : SQ_ERR_CUDA;
}
