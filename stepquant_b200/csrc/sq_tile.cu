// Generic tile kernel: one CTA of 256 threads per (request, value head).
//
// The whole [K, V] state tile lives in shared memory as fp32, so every
// supported shape (K, V in 4..128) and every plan (GDN incl. 2-bit and fp16
// pivot heads, KDA with mixed per-row widths and fp16 pivot rows) runs through
// one code path.  The ordered sums of fit_state are evaluated by one thread
// per row / column in torch's CPU order, which makes the page bytes identical
// to the reference quantizer's.  The register-resident kernel in sq_fast.cu
// covers the K = V = 128 GDN heads of the benchmark and must produce the same
// bytes; this kernel is its cross-check.
#include "sq_tile.cuh"

namespace sq {

namespace {

struct Smem {
    float *xs;    // [K*V] state tile
    int8_t *zq;   // [K*V] integer levels
    int *rbits;   // [K]
    int *roff;    // [K]
    int *rrow;    // [K]
    float *rw;    // [K] impact
    float *rr;    // [K] row scale r (old, then new)
    float *qv;    // [K]
    float *kv;    // [K]
    float *dec;   // [K] decay
    float *cold;  // [V] stored column scale
    float *c0;    // [V]
    float *c1;    // [V]
    float *del;   // [V] delta
    float *vin;   // [V] value input, then readout
    float *red;   // [32]
    float *r2s;   // [K * groups] GDN 2-bit value-group row scales
};

__device__ Smem carve(unsigned char *raw, int K, int V, int groups) {
    Smem s;
    s.xs = reinterpret_cast<float *>(raw);
    s.zq = reinterpret_cast<int8_t *>(s.xs + K * V);
    s.rbits = reinterpret_cast<int *>(s.zq + K * V);
    s.roff = s.rbits + K;
    s.rrow = s.roff + K;
    s.rw = reinterpret_cast<float *>(s.rrow + K);
    s.rr = s.rw + K;
    s.qv = s.rr + K;
    s.kv = s.qv + K;
    s.dec = s.kv + K;
    s.cold = s.dec + K;
    s.c0 = s.cold + V;
    s.c1 = s.c0 + V;
    s.del = s.c1 + V;
    s.vin = s.del + V;
    s.red = s.vin + V;
    s.r2s = s.red + 32;
    (void)groups;
    return s;
}

}  // namespace

size_t tile_smem_bytes(int K, int V, int groups) {
    return size_t(K) * V * 5 + size_t(K) * 9 * 4 + size_t(V) * 5 * 4 + 32 * 4 + size_t(K) * groups * 4;
}

// Fit one (request, head) tile to a baseline format and store its page bytes
// (formats.py:51-82 group_fit / dual_fit, format_pool.py:9-27 layout): the
// symmetric format's per-group scale fp16(absmax / limit) with zero point
// `limit`; DSQ's row scale r = fp16(sqrt(max(mean |x|, 1e-20))) (torch's row
// sum order), column scale c = fp16(max_k |x / r| / levels) and codes
// rint(x / r / c); every division correctly rounded.  Codes go to each row's
// bitstream as level + limit.
__device__ void format_store(int fmt, int G, uint8_t *page, Smem &s, int K, int V, int coff, int tid) {
    const int groups = V / G;
    for (int k = tid; k < K; k += kThreads) {
        const float *row = s.xs + k * V;
        const float limit = float((1 << (s.rbits[k] - 1)) - 1);
        if (fmt == 2) {
            for (int g = 0; g < groups; ++g) {
                float m = 0.f;
                for (int i = 0; i < G; ++i) m = fmaxf(m, fabsf(row[g * G + i]));
                const float sc = fp16_scale(__fdiv_rn(m, limit));
                s.r2s[k * groups + g] = sc;
                put_half(page, s.rrow[k] + 4 * g, sc);
                put_half(page, s.rrow[k] + 4 * g + 2, limit);
            }
        } else {
            const float sum = torch_inner_sum(V, [&](int i) { return fabsf(row[i]); });
            const float r = fp16_scale(__fsqrt_rn(fmaxf(__fdiv_rn(sum, float(V)), 1e-20f)));
            s.rr[k] = r;
            put_half(page, s.rrow[k], r);
        }
    }
    __syncthreads();
    if (fmt == 3) {
        for (int v = tid; v < V; v += kThreads) {
            float m = 0.f;
            for (int k = 0; k < K; ++k) {
                const float limit = float((1 << (s.rbits[k] - 1)) - 1);
                m = fmaxf(m, __fdiv_rn(fabsf(__fdiv_rn(s.xs[k * V + v], s.rr[k])), limit));
            }
            const float c = fp16_scale(m);
            s.c1[v] = c;
            put_half(page, coff + 4 * v, c);
            put_half(page, coff + 4 * v + 2, 0.f);
        }
        __syncthreads();
    }
    for (int e = tid; e < K * V; e += kThreads) {
        const int k = e / V, v = e % V;
        const float limit = float((1 << (s.rbits[k] - 1)) - 1);
        const float y = fmt == 2 ? __fdiv_rn(s.xs[e], s.r2s[k * groups + v / G])
                                 : __fdiv_rn(__fdiv_rn(s.xs[e], s.rr[k]), s.c1[v]);
        s.zq[e] = int8_t(fminf(fmaxf(rintf(y), -limit), limit));
    }
    __syncthreads();
    for (int k = tid; k < K; k += kThreads) {  // one thread per row bitstream
        const int b = s.rbits[k], off = (1 << (b - 1)) - 1;
        uint8_t *dst = page + s.roff[k];
        uint32_t acc = 0;
        int nbits = 0, w = 0;
        for (int v = 0; v < V; ++v) {
            acc |= uint32_t(int(s.zq[k * V + v]) + off) << nbits;
            nbits += b;
            while (nbits >= 8) {
                dst[w++] = uint8_t(acc & 0xffu);
                acc >>= 8;
                nbits -= 8;
            }
        }
        if (nbits > 0) dst[w] = uint8_t(acc & 0xffu);  // 3/5-bit KDA chunks: zero tail bits
    }
}

template <int MODE>
__global__ void __launch_bounds__(kThreads) tile_kernel(TileParams p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const sq_plan &P = p.plan;
    const int H = P.heads, K = P.keys, V = P.values;
    const bool kda = P.architecture == SQ_KDA;
    const int G = P.value_group_size;
    const int groups = kda ? 1 : V / G;
    const int tid = threadIdx.x;
    const int req = blockIdx.x / H;
    const int head = blockIdx.x % H;
    Smem s = carve(smem_raw, K, V, groups);
    const int64_t tile_index = (int64_t(req) * H + head) * K * V;

    // ---- request slot ----------------------------------------------------
    int64_t slot = 1;
    if (MODE != kFit) slot = p.slots[req];
    if (MODE == kReadout && head == 0 && tid == 0) p.stable_slots[req] = slot;
    if (p.skip_fast && fast_head_dev(P, head)) return;
    if (p.skip_pivot && P.bits[head * P.keys] == 16) return;
    if (p.skip_two && P.bits[head * P.keys] == 2) return;
    bool active = slot > 0;
    if (active && MODE != kFit && slot >= p.num_slots) {
        if (head == 0 && tid == 0) flag(p.status, SQ_STATUS_SLOT_RANGE);
        active = false;
    }
    if (!active) {
        if (MODE == kDecode) {
            for (int e = tid; e < K * V; e += kThreads) p.dense_out[tile_index + e] = 0.f;
        }
        if (MODE == kStep || MODE == kReadout) {
            for (int v = tid; v < V; v += kThreads)
                store_from_float(p.step.out, p.step.io_dtype, (int64_t(req) * H + head) * V + v, 0.f);
            if (MODE == kStep && p.dense_out)
                for (int e = tid; e < K * V; e += kThreads) p.dense_out[tile_index + e] = 0.f;
        }
        return;
    }
    uint8_t *page = MODE == kFit ? nullptr : p.pages + slot * P.page_bytes;

    // ---- head metadata ---------------------------------------------------
    for (int k = tid; k < K; k += kThreads) {
        s.rbits[k] = P.bits[head * K + k];
        s.roff[k] = P.offsets[head * K + k];
        s.rrow[k] = P.rows[head * K + k];
        s.rw[k] = P.impact[head * K + k];
    }
    const int stride = P.offsets[H * K + head];
    const int coff = P.columns[head];
    const int tile = min(kda ? 4 : 16, V);
    const bool bytes = P.storage == 1;  // byte carriers (pool.py:29-43): codes at code_base + k + v K
    const int fmt = P.storage >= 2 ? P.storage : 0;  // baseline formats: 2 symmetric groups, 3 dual axis (DSQ)
    const bool gdn2 = !kda && P.bits[head * K] == 2;
    if (MODE == kWriteback && coff < 0) return;  // all-pivot head: finished by sq_readout
    __syncthreads();

    // ---- load the state ----------------------------------------------------
    if (MODE == kEncode || MODE == kFit) {
        for (int e = tid; e < K * V; e += kThreads) s.xs[e] = p.dense_in[tile_index + e];
    } else if (fmt) {
        // Baseline formats (format_pool.py:77-128 read, formats.py:51-82): each row one little-endian
        // bitstream; symmetric (code - zero) * scale per value group, DSQ
        // (r c)(code - levels).  No pivot rows.
        const int G = P.value_group_size;
        for (int e = tid; e < K * V; e += kThreads) {
            const int k = e / V, v = e % V;
            const int b = s.rbits[k];
            const float code = float(read_code(page + s.roff[k], uint32_t(v * b), b));
            float x;
            if (fmt == 2) {
                const int64_t meta = s.rrow[k] + 4 * int64_t(v / G);
                x = __fmul_rn(__fsub_rn(code, half_at(page, meta + 2)), half_at(page, meta));
            } else {
                const float rc = __fmul_rn(half_at(page, s.rrow[k]), half_at(page, coff + 4 * v));
                x = __fmul_rn(rc, __fsub_rn(code, float((1 << (b - 1)) - 1)));
            }
            s.xs[e] = x;
        }
    } else {
        for (int v = tid; v < V; v += kThreads) s.cold[v] = coff >= 0 ? half_at(page, coff + 2 * v) : 0.f;
        for (int k = tid; k < K; k += kThreads) {
            const int b = s.rbits[k];
            if (b == 16) continue;
            if (gdn2) {
                for (int g = 0; g < groups; ++g) s.r2s[k * groups + g] = half_at(page, s.rrow[k] + 2 * g);
            } else {
                s.rr[k] = half_at(page, s.rrow[k]);
            }
        }
        __syncthreads();
        for (int e = tid; e < K * V; e += kThreads) {
            const int k = e / V, v = e % V;
            const int b = s.rbits[k];
            float x;
            if (b == 16) {
                x = MODE == kWriteback ? 0.f : half_at(page, pivot_at(s.roff[k], v, tile, stride, bytes));
            } else {
                // byte carriers: the signed level (KDA: times 2^(8-b)) at code_base + k + v K
                const float z = bytes ? float(reinterpret_cast<const int8_t *>(page)[s.roff[k] + int64_t(v) * K])
                                      : level_of(read_code(page + s.roff[k] + int64_t(v / tile) * stride,
                                                           uint32_t((v % tile) * b), b), b, kda);
                const float r = gdn2 ? s.r2s[k * groups + v / G] : s.rr[k];
                x = __fmul_rn(__fmul_rn(r, s.cold[v]), z);
            }
            s.xs[e] = x;
        }
    }
    if (MODE == kDecode) {
        __syncthreads();
        for (int e = tid; e < K * V; e += kThreads) p.dense_out[tile_index + e] = s.xs[e];
        return;
    }

    // ---- recurrent update ----------------------------------------------------
    if (MODE == kStep || MODE == kReadout || MODE == kWriteback) {
        float beta = 0.f;
        if (MODE == kWriteback) {
            const float *sc = p.scratch + int64_t(req) * p.scratch_stride + int64_t(head) * (V + 2 * K);
            for (int v = tid; v < V; v += kThreads) s.del[v] = sc[v];
            for (int k = tid; k < K; k += kThreads) {
                s.kv[k] = sc[V + k];
                s.dec[k] = sc[V + K + k];
            }
        } else {
            const sq_step_args &a = p.step;
            const int qh = head / (H / a.qk_heads);
            float qq = 0.f, kk = 0.f;
            for (int k = tid; k < K; k += kThreads) {
                const float qx = load_as_float(a.q, a.io_dtype, int64_t(req) * a.q_stride + int64_t(qh) * K + k);
                const float kx = load_as_float(a.k, a.io_dtype, int64_t(req) * a.k_stride + int64_t(qh) * K + k);
                s.qv[k] = qx;
                s.kv[k] = kx;
                qq = fmaf(qx, qx, qq);
                kk = fmaf(kx, kx, kk);
            }
            if (a.normalize) {
                const float qn = __frsqrt_rn(block_sum(qq, s.red) + 1e-6f);
                const float kn = __frsqrt_rn(block_sum(kk, s.red) + 1e-6f);
                for (int k = tid; k < K; k += kThreads) {
                    s.qv[k] *= qn;
                    s.kv[k] *= kn;
                }
            }
            for (int k = tid; k < K; k += kThreads) s.qv[k] *= a.scale;
            float braw = load_as_float(a.beta, a.gate_dtype, int64_t(req) * H + head);
            beta = a.a_log ? 1.f / (1.f + expf(-braw)) : braw;
            const float neg_a = a.a_log ? -expf(a.a_log[head]) : 0.f;
            for (int k = tid; k < K; k += kThreads) {
                const int64_t gi = kda ? (int64_t(req) * H + head) * K + k : int64_t(req) * H + head;
                float g = load_as_float(a.g, a.gate_dtype, gi);
                if (a.a_log) {
                    const float u = g + a.dt_bias[kda ? head * K + k : head];
                    g = neg_a * (u > 20.f ? u : logf(1.f + expf(fminf(u, 20.f))));
                }
                s.dec[k] = expf(g);
            }
            for (int v = tid; v < V; v += kThreads)
                s.vin[v] = load_as_float(a.v, a.io_dtype, int64_t(req) * a.v_stride + int64_t(head) * V + v);
        }
        __syncthreads();
        for (int e = tid; e < K * V; e += kThreads) s.xs[e] = __fmul_rn(s.xs[e], s.dec[e / V]);
        __syncthreads();
        if (MODE != kWriteback) {
            for (int v = tid; v < V; v += kThreads) {
                float acc = 0.f;
                for (int k = 0; k < K; ++k) acc = fmaf(s.kv[k], s.xs[k * V + v], acc);
                s.del[v] = __fmul_rn(beta, __fsub_rn(s.vin[v], acc));
            }
            __syncthreads();
        }
        for (int e = tid; e < K * V; e += kThreads) {
            const int k = e / V, v = e % V;
            if (MODE == kWriteback && s.rbits[k] == 16) continue;
            s.xs[e] = __fadd_rn(s.xs[e], __fmul_rn(s.kv[k], s.del[v]));
        }
        __syncthreads();
        if (MODE != kWriteback) {
            const sq_step_args &a = p.step;
            for (int v = tid; v < V; v += kThreads) {
                float acc = 0.f;
                for (int k = 0; k < K; ++k) acc = fmaf(s.qv[k], s.xs[k * V + v], acc);
                store_from_float(a.out, a.io_dtype, (int64_t(req) * H + head) * V + v, acc);
            }
        }
        if (MODE == kStep && p.dense_out)
            for (int e = tid; e < K * V; e += kThreads) p.dense_out[tile_index + e] = s.xs[e];
        if (MODE == kReadout) {
            float *sc = p.scratch + int64_t(req) * p.scratch_stride + int64_t(head) * (V + 2 * K);
            for (int v = tid; v < V; v += kThreads) sc[v] = s.del[v];
            for (int k = tid; k < K; k += kThreads) {
                sc[V + k] = s.kv[k];
                sc[V + K + k] = s.dec[k];
            }
            // fp16 pivot rows are final: store them now (readout.py:118-121).
            for (int e = tid; e < K * V; e += kThreads) {
                const int k = e / V, v = e % V;
                if (s.rbits[k] != 16) continue;
                put_half(page, pivot_at(s.roff[k], v, tile, stride, bytes), s.xs[e]);
            }
            return;
        }
        if (MODE == kStep && coff < 0) {
            // All-pivot head: no quantization, store the fp16 rows.
            for (int e = tid; e < K * V; e += kThreads) {
                const int k = e / V, v = e % V;
                put_half(page, pivot_at(s.roff[k], v, tile, stride, bytes), s.xs[e]);
            }
            return;
        }
    }
    if (MODE == kEncode && coff < 0) {
        __syncthreads();
        for (int e = tid; e < K * V; e += kThreads) {
            const int k = e / V, v = e % V;
            put_half(page, pivot_at(s.roff[k], v, tile, stride, bytes), s.xs[e]);
        }
        return;
    }
    __syncthreads();
    if (fmt) {
        format_store(fmt, P.value_group_size, page, s, K, V, coff, tid);
        return;
    }

    // ---- fit_state (quantization.py:54-98) ----------------------------------
    // Row scales r = fp16(sqrt(max(mean|x|, 1e-20) / w)).
    for (int k = tid; k < K; k += kThreads) {
        const float *row = s.xs + k * V;
        const float sum = torch_inner_sum(V, [&](int i) { return fabsf(row[i]); });
        const float mean = __fdiv_rn(sum, float(V));
        s.rr[k] = fp16_scale(__fsqrt_rn(__fdiv_rn(fmaxf(mean, 1e-20f), s.rw[k])));
        if (gdn2) {
            for (int g = 0; g < groups; ++g) {
                const float gs = torch_inner_sum(G, [&](int i) { return fabsf(row[g * G + i]); });
                const float gm = __fdiv_rn(gs, float(G));
                s.r2s[k * groups + g] = fp16_scale(__fsqrt_rn(__fdiv_rn(fmaxf(gm, 1e-20f), s.rw[k])));
            }
        }
    }
    __syncthreads();
    auto rfull = [&](int k, int v) { return gdn2 ? s.r2s[k * groups + v / G] : s.rr[k]; };
    // Initial column scale: c = fp16(max_k |x/r| / (qmax * norm)) over integer rows.
    for (int v = tid; v < V; v += kThreads) {
        float m = 0.f;
        for (int k = 0; k < K; ++k) {
            const int b = s.rbits[k];
            if (b == 16) continue;
            const float sc = __fdiv_rn(s.xs[k * V + v], rfull(k, v));
            const float lim = __fmul_rn(qmax_of(b, !kda), norm_of(b, kda));
            m = fmaxf(m, __fdiv_rn(fabsf(sc), lim));
        }
        s.c0[v] = fp16_scale(m);
    }
    __syncthreads();
    auto encode = [&](const float *cols) {
        for (int e = tid; e < K * V; e += kThreads) {
            const int k = e / V, v = e % V;
            const int b = s.rbits[k];
            const float sc = __fdiv_rn(s.xs[e], rfull(k, v));
            const float y = __fdiv_rn(__fdiv_rn(sc, cols[v]), norm_of(b, kda));
            float z;
            if (gdn2) {
                z = (y >= 0.f ? 1.f : -1.f) * (fabsf(y) >= 2.f ? 3.f : 1.f);
            } else {
                const float qm = qmax_of(b, !kda);
                z = fminf(fmaxf(rintf(y), -qm), qm);
            }
            s.zq[e] = int8_t(z);
        }
    };
    encode(s.c0);
    __syncthreads();
    // One weighted least-squares refit of c (torch's column-sum order).
    for (int j = tid; j < 2 * kMaxDim; j += kThreads) {
        const int v = j % kMaxDim;
        const bool den = j >= kMaxDim;
        if (v >= V) continue;
        const float total = torch_outer_sum(K, V, [&](int k) {
            const int b = s.rbits[k];
            if (b == 16) return 0.f;
            const float w2 = __fmul_rn(s.rw[k], s.rw[k]);
            const float vq = __fmul_rn(__fmul_rn(rfull(k, v), norm_of(b, kda)), float(s.zq[k * V + v]));
            return den ? __fmul_rn(w2, __fmul_rn(vq, vq)) : __fmul_rn(__fmul_rn(w2, vq), s.xs[k * V + v]);
        });
        if (den) s.c1[v] = total; else s.del[v] = total;  // del reused: numerator
    }
    __syncthreads();
    for (int v = tid; v < V; v += kThreads) {
        const float num = s.del[v], den = s.c1[v];
        s.c1[v] = den > 0.f ? fp16_scale(__fdiv_rn(num, fmaxf(den, 1e-30f))) : s.c0[v];
    }
    __syncthreads();
    encode(s.c1);
    __syncthreads();

    // ---- outputs ------------------------------------------------------------
    if (MODE == kFit) {
        for (int e = tid; e < K * V; e += kThreads) {
            const int k = e / V, v = e % V;
            const int b = s.rbits[k];
            const float z = float(s.zq[e]);
            p.fit_z[tile_index + e] = int16_t(s.zq[e]);
            if (p.fit_recon) {
                float rec;
                if (b == 16) {
                    rec = __half2float(__float2half_rn(s.xs[e]));
                } else {
                    rec = __fmul_rn(__fmul_rn(__fmul_rn(rfull(k, v), s.c1[v]), norm_of(b, kda)), z);
                }
                p.fit_recon[tile_index + e] = rec;
            }
        }
        for (int k = tid; k < K; k += kThreads) p.fit_r[(int64_t(req) * H + head) * K + k] = half_bits(s.rr[k]);
        for (int v = tid; v < V; v += kThreads) p.fit_c[(int64_t(req) * H + head) * V + v] = half_bits(s.c1[v]);
        if (gdn2 && p.fit_r2) {
            int h2 = 0, n2 = 0;
            for (int h = 0; h < H; ++h) {
                const bool two = P.bits[h * K] == 2;
                h2 += (two && h < head);
                n2 += two;
            }
            for (int j = tid; j < K * groups; j += kThreads)
                p.fit_r2[((int64_t(req) * n2 + h2) * K) * groups + j] = half_bits(s.r2s[j]);
        }
        return;
    }
    // Page stores: codes of integer rows, fp16 pivots, r, c.
    const int tiles = V / tile;
    if (bytes) {
        for (int e = tid; e < K * V; e += kThreads) {
            const int k = e / V, v = e % V;
            const int b = s.rbits[k];
            if (b == 16) {
                if (MODE != kWriteback) put_half(page, pivot_at(s.roff[k], v, tile, stride, bytes), s.xs[e]);
                continue;
            }
            const int z = int(s.zq[e]) * (kda ? (1 << (8 - b)) : 1);  // fit.py:111-115
            reinterpret_cast<int8_t *>(page)[s.roff[k] + int64_t(v) * K] = int8_t(z);
        }
    }
    for (int ch = tid; !bytes && ch < K * tiles; ch += kThreads) {
        const int k = ch / tiles, t = ch % tiles;
        const int b = s.rbits[k];
        uint8_t *dst = page + s.roff[k] + int64_t(t) * stride;
        if (b == 16) {
            if (MODE == kWriteback) continue;
            for (int u = 0; u < tile; ++u) put_half(dst, 2 * u, s.xs[k * V + t * tile + u]);
            continue;
        }
        uint64_t acc = 0;
        int nbits = 0, w = 0;
        for (int u = 0; u < tile; ++u) {
            acc |= uint64_t(code_of(float(s.zq[k * V + t * tile + u]), b, kda)) << nbits;
            nbits += b;
            while (nbits >= 8) {
                dst[w++] = uint8_t(acc & 0xffu);
                acc >>= 8;
                nbits -= 8;
            }
        }
        if (nbits > 0) dst[w] = uint8_t(acc & 0xffu);  // 3/5-bit KDA chunks: zero tail bits
    }
    for (int k = tid; k < K; k += kThreads) {
        if (s.rbits[k] == 16) continue;
        if (gdn2) {
            for (int g = 0; g < groups; ++g) put_half(page, s.rrow[k] + 2 * g, s.r2s[k * groups + g]);
        } else {
            put_half(page, s.rrow[k], s.rr[k]);
        }
    }
    if (coff >= 0)
        for (int v = tid; v < V; v += kThreads) put_half(page, coff + 2 * v, s.c1[v]);
}

template <int MODE>
cudaError_t launch_tile_mode(const TileParams &p, int items, cudaStream_t stream) {
    const int groups = p.plan.architecture == SQ_KDA ? 1 : p.plan.values / p.plan.value_group_size;
    const size_t smem = tile_smem_bytes(p.plan.keys, p.plan.values, groups);
    cudaError_t err = cudaFuncSetAttribute(tile_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (err != cudaSuccess) return err;
    tile_kernel<MODE><<<items, kThreads, smem, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_tile(int mode, const TileParams &p, int items, cudaStream_t stream) {
    if (items <= 0) return cudaSuccess;
    switch (mode) {
        case kEncode: return launch_tile_mode<kEncode>(p, items, stream);
        case kDecode: return launch_tile_mode<kDecode>(p, items, stream);
        case kStep: return launch_tile_mode<kStep>(p, items, stream);
        case kReadout: return launch_tile_mode<kReadout>(p, items, stream);
        case kWriteback: return launch_tile_mode<kWriteback>(p, items, stream);
        case kFit: return launch_tile_mode<kFit>(p, items, stream);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace sq
