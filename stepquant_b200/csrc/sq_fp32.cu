// FP32 state-pool decode step (the reference's FP32 baseline,
// stepquant/kernels/floating.py:20-53): same gated delta rule and readout on
// an uncompressed fp32 state [num_slots, H, K, V], updated in place.
// One CTA per (request, head); each column's K state values are held in the
// registers of K/64 threads (one for K <= 64), so the state is read once and
// written once.
#include <cuda_runtime.h>

#include "sq_common.cuh"

namespace sq {

template <int K>
__global__ void __launch_bounds__(256) fp32_step_kernel(float *state, int64_t num_slots, int H, int V, int kda,
                                                        const int64_t *slots, sq_step_args a, int32_t *status) {
    // Thread (slice, v) keeps rows [slice*RP, slice*RP + RP) of column v in registers.
    constexpr int RP = K > 64 ? 64 : K;
    constexpr int S = K / RP;
    __shared__ float qs[K], ks[K], ds[K], red[64], part[2][S][128];
    const int req = blockIdx.x / H, head = blockIdx.x % H;
    const int tid = threadIdx.x;
    int64_t slot = slots[req];
    bool active = slot > 0;
    if (active && slot >= num_slots) {
        if (head == 0 && tid == 0) flag(status, SQ_STATUS_SLOT_RANGE);
        active = false;
    }
    if (!active) {
        for (int v = tid; v < V; v += blockDim.x) store_from_float(a.out, a.io_dtype, (int64_t(req) * H + head) * V + v, 0.f);
        return;
    }
    const int qh = head / (H / a.qk_heads);
    float qq = 0.f, kk = 0.f;
    for (int k = tid; k < K; k += blockDim.x) {
        const float qx = load_as_float(a.q, a.io_dtype, int64_t(req) * a.q_stride + int64_t(qh) * K + k);
        const float kx = load_as_float(a.k, a.io_dtype, int64_t(req) * a.k_stride + int64_t(qh) * K + k);
        qs[k] = qx;
        ks[k] = kx;
        qq = fmaf(qx, qx, qq);
        kk = fmaf(kx, kx, kk);
    }
    float qn = 1.f, kn = 1.f;
    if (a.normalize) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            qq += __shfl_xor_sync(0xffffffffu, qq, o);
            kk += __shfl_xor_sync(0xffffffffu, kk, o);
        }
        if ((tid & 31) == 0) {
            red[tid >> 5] = qq;
            red[32 + (tid >> 5)] = kk;
        }
        __syncthreads();
        float tq = 0.f, tk = 0.f;
        for (int w = 0; w < int(blockDim.x) / 32; ++w) {
            tq += red[w];
            tk += red[32 + w];
        }
        qn = __frsqrt_rn(tq + 1e-6f);
        kn = __frsqrt_rn(tk + 1e-6f);
    }
    const float braw = load_as_float(a.beta, a.gate_dtype, int64_t(req) * H + head);
    const float beta = a.a_log ? 1.f / (1.f + expf(-braw)) : braw;
    const float neg_a = a.a_log ? -expf(a.a_log[head]) : 0.f;
    __syncthreads();
    for (int k = tid; k < K; k += blockDim.x) {
        qs[k] = qs[k] * qn * a.scale;
        ks[k] = ks[k] * kn;
        const int64_t gi = kda ? (int64_t(req) * H + head) * K + k : int64_t(req) * H + head;
        float g = load_as_float(a.g, a.gate_dtype, gi);
        if (a.a_log) {
            const float u = g + a.dt_bias[kda ? head * K + k : head];
            g = neg_a * (u > 20.f ? u : logf(1.f + expf(fminf(u, 20.f))));
        }
        ds[k] = expf(g);
    }
    __syncthreads();
    const int v = tid % V, slice = tid / V;
    const bool mine = slice < S;
    float *col = state + ((slot * H + head) * int64_t(K) + slice * RP) * V + v;
    float x[RP];
    float acc = 0.f;
    if (mine) {
#pragma unroll
        for (int k = 0; k < RP; ++k) {
            x[k] = __fmul_rn(col[int64_t(k) * V], ds[slice * RP + k]);
            acc = fmaf(ks[slice * RP + k], x[k], acc);
        }
        part[0][slice][v] = acc;
    }
    __syncthreads();
    if (mine) {
        float kx = 0.f;
#pragma unroll
        for (int j = 0; j < S; ++j) kx += part[0][j][v];
        const float vin = load_as_float(a.v, a.io_dtype, int64_t(req) * a.v_stride + int64_t(head) * V + v);
        const float delta = __fmul_rn(beta, __fsub_rn(vin, kx));
        float out = 0.f;
#pragma unroll
        for (int k = 0; k < RP; ++k) {
            x[k] = __fadd_rn(x[k], __fmul_rn(ks[slice * RP + k], delta));
            out = fmaf(qs[slice * RP + k], x[k], out);
            col[int64_t(k) * V] = x[k];
        }
        part[1][slice][v] = out;
    }
    __syncthreads();
    if (mine && slice == 0) {
        float out = 0.f;
#pragma unroll
        for (int j = 0; j < S; ++j) out += part[1][j][v];
        store_from_float(a.out, a.io_dtype, (int64_t(req) * H + head) * V + v, out);
    }
}

cudaError_t launch_fp32_step(float *state, int64_t num_slots, int H, int K, int V, int kda, const int64_t *slots,
                             int batch, const sq_step_args &a, int32_t *status, cudaStream_t stream) {
    if (batch <= 0) return cudaSuccess;
    const int slices = K > 64 ? K / 64 : 1;
    int threads = V * slices;
    threads = threads < 32 ? 32 : threads;
    const int grid = batch * H;
    switch (K) {
        case 4: fp32_step_kernel<4><<<grid, threads, 0, stream>>>(state, num_slots, H, V, kda, slots, a, status); break;
        case 8: fp32_step_kernel<8><<<grid, threads, 0, stream>>>(state, num_slots, H, V, kda, slots, a, status); break;
        case 16: fp32_step_kernel<16><<<grid, threads, 0, stream>>>(state, num_slots, H, V, kda, slots, a, status); break;
        case 32: fp32_step_kernel<32><<<grid, threads, 0, stream>>>(state, num_slots, H, V, kda, slots, a, status); break;
        case 64: fp32_step_kernel<64><<<grid, threads, 0, stream>>>(state, num_slots, H, V, kda, slots, a, status); break;
        case 128: fp32_step_kernel<128><<<grid, threads, 0, stream>>>(state, num_slots, H, V, kda, slots, a, status); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace sq
