// extern "C" entry points of libstepquant_b200 (declared in include/stepquant_b200.h).
// Host-side argument validation mirrors the reference's eager ValueErrors
// (stepquant/kernels/pool.py:71-84,186-187,210-230; quantization.py:14-26)
// and returns an sq_error code instead of raising.
#include <cuda_runtime.h>

#include <vector>

#include "sq_tile.cuh"

namespace sq {
cudaError_t launch_pack(const int16_t *codes, int64_t n, int bits, uint8_t *out, cudaStream_t stream);
cudaError_t launch_unpack(const uint8_t *data, int64_t count, int bits, int16_t *out, cudaStream_t stream);
int64_t packed_bytes(int64_t n, int bits);
cudaError_t launch_fp32_step(float *state, int64_t num_slots, int H, int K, int V, int kda, const int64_t *slots,
                             int batch, const sq_step_args &a, int32_t *status, cudaStream_t stream);
cudaError_t launch_division_selftest(const float *a, const uint16_t *b, float *out, int64_t n, cudaStream_t stream);
}  // namespace sq

namespace {

bool pow2_dim(int32_t x) { return x >= 4 && x <= sq::kMaxDim && (x & (x - 1)) == 0; }

int32_t check_plan(const sq_plan *p) {
    if (!p || !p->bits || !p->impact || !p->offsets || !p->rows || !p->columns) return SQ_ERR_ARGUMENT;
    if (p->architecture != SQ_GDN && p->architecture != SQ_KDA) return SQ_ERR_ARGUMENT;
    if (p->heads < 1 || p->page_bytes < 2 || p->value_group_size < 1) return SQ_ERR_ARGUMENT;
    if (p->storage < 0 || p->storage > 3) return SQ_ERR_ARGUMENT;  // packed, byte, symmetric, DSQ
    if (!pow2_dim(p->keys) || !pow2_dim(p->values)) return SQ_ERR_SHAPE;
    if (p->architecture == SQ_GDN) {
        if (p->values % p->value_group_size) return SQ_ERR_SHAPE;
        if (p->values / p->value_group_size > sq::kMaxGroups) return SQ_ERR_UNSUPPORTED;
    }
    return SQ_OK;
}

}  // namespace

namespace sq {
// Plan validation for the other translation units of the library.
int32_t validate_plan(const sq_plan *p) { return check_plan(p); }
}  // namespace sq

namespace {

int32_t check_step(const sq_plan *p, const sq_step_args *a) {
    if (!a || !a->q || !a->k || !a->v || !a->g || !a->beta || !a->out) return SQ_ERR_ARGUMENT;
    if (a->io_dtype < SQ_F32 || a->io_dtype > SQ_F16 || a->gate_dtype < SQ_F32 || a->gate_dtype > SQ_F16)
        return SQ_ERR_ARGUMENT;
    if (a->q_stride < 0 || a->k_stride < 0 || a->v_stride < 0) return SQ_ERR_SHAPE;
    if (a->qk_heads < 1 || p->heads % a->qk_heads) return SQ_ERR_SHAPE;
    if (a->a_log && !a->dt_bias) return SQ_ERR_ARGUMENT;
    return SQ_OK;
}

int32_t cuda_status(cudaError_t e) { return e == cudaSuccess ? SQ_OK : SQ_ERR_CUDA; }

sq::TileParams base_params(const sq_plan *plan, uint8_t *pages, int64_t num_slots, const int64_t *slots,
                           int32_t *status) {
    sq::TileParams t{};
    t.plan = *plan;
    t.pages = pages;
    t.num_slots = num_slots;
    t.slots = slots;
    t.status = status;
    return t;
}

// Step, readout and writeback go to the register-resident kernels for the heads
// they handle (GDN, K = V = 128, widths 4/6/8; KDA, K = V = 128, code region
// within the stage buffer) and to the tile kernel for the rest; with a host copy of the bits the tile launch is skipped when no head
// needs it.  Every other mode runs on the tile kernel.
// Host restatement of the KDA head test of fast_head_dev from a head's bits
// (the packed layout's value-tile stride, tile 4).
bool kda_head_fast_host(const int32_t *bits, int keys, int values) {
    int64_t local = 0;
    bool any_int = false;
    for (int k = 0; k < keys; ++k) {
        if (bits[k] == 16) local = (local + 1) / 2 * 2;
        else any_int = true;
        local += (4 * bits[k] + 7) / 8;
    }
    return sq::kda_head_fits((local + 1) / 2 * 2, values, any_int ? 0 : -1);
}

int32_t run(int mode, sq::TileParams t, int32_t batch, cudaStream_t stream) {
    const int items = batch * t.plan.heads;
    if (items <= 0) return SQ_OK;
    const bool fast_mode = mode == sq::kStep || mode == sq::kReadout || mode == sq::kWriteback;
    const bool gdn_codec = mode == sq::kEncode || mode == sq::kDecode;
    if (fast_mode && sq::kda_fast_eligible(t.plan)) {
        if (cudaError_t e = sq::launch_fast_kda(mode, t, batch, stream)) return cuda_status(e);
        bool rest = true;
        if (t.plan.bits_host) {
            rest = false;
            for (int h = 0; h < t.plan.heads; ++h)
                rest = rest || !kda_head_fast_host(t.plan.bits_host + h * t.plan.keys, t.plan.keys, t.plan.values);
        }
        if (!rest) return SQ_OK;
        t.skip_fast = 1;
    } else if ((fast_mode || gdn_codec) && sq::fast_eligible(t.plan, t.pages)) {
        if (cudaError_t e = sq::launch_fast(mode, t, batch, stream)) return cuda_status(e);
        sq::PivotHeads ph;
        sq::TwoHeads th;
        const bool pivots = sq::pivot_heads(t.plan, &ph);  // pivot and 2-bit heads run in launch_fast
        const bool twos = sq::two_heads(t.plan, &th);
        bool rest = true;
        if (t.plan.bits_host) {
            rest = false;
            for (int h = 0; h < t.plan.heads; ++h) {
                const int width = t.plan.bits_host[h * t.plan.keys];
                rest = rest || !(sq::fast_head(t.plan, width) || (pivots && width == 16) || (twos && width == 2));
            }
        }
        if (!rest) return SQ_OK;
        t.skip_fast = 1;
        t.skip_pivot = pivots ? 1 : 0;
        t.skip_two = twos ? 1 : 0;
    }
    return cuda_status(sq::launch_tile(mode, t, items, stream));
}

}  // namespace

extern "C" {

int32_t sq_version(void) { return 100; }

const char *sq_error_string(int32_t code) {
    switch (code) {
        case SQ_OK: return "ok";
        case SQ_ERR_ARGUMENT: return "invalid argument";
        case SQ_ERR_SHAPE: return "invalid shape, stride or head grouping";
        case SQ_ERR_UNSUPPORTED: return "configuration not supported by this build";
        case SQ_ERR_CUDA: return "CUDA launch failure";
        case SQ_ERR_CAPACITY: return "batch exceeds the scratch capacity";
        default: return "unknown error";
    }
}

int32_t sq_packed_layout(int32_t architecture, int32_t heads, int32_t keys, int32_t values,
                         int32_t value_group_size, const int32_t *bits, int32_t storage, int32_t *offsets_out,
                         int32_t *rows_out, int32_t *columns_out, int64_t *page_bytes_out) {
    if (!bits || !offsets_out || !rows_out || !columns_out || !page_bytes_out) return SQ_ERR_ARGUMENT;
    if ((architecture != SQ_GDN && architecture != SQ_KDA) || heads < 1 || keys < 1 || values < 1 ||
        value_group_size < 1 || (storage != 0 && storage != 1))
        return SQ_ERR_ARGUMENT;
    const bool kda = architecture == SQ_KDA;
    for (int i = 0; i < heads * keys; ++i) {
        const int b = bits[i];
        if (b != 2 && b != 3 && b != 4 && b != 5 && b != 6 && b != 8 && b != 16) return SQ_ERR_ARGUMENT;
    }
    auto head_has_int = [&](int h) {
        for (int k = 0; k < keys; ++k)
            if (bits[h * keys + k] != 16) return true;
        return false;
    };
    int64_t cursor = 0;
    const int tile = values < (kda ? 4 : 16) ? values : (kda ? 4 : 16);
    std::vector<int64_t> strides(heads);
    int n = 0;
    if (storage == 1) {
        for (int h = 0; h < heads; ++h) {
            const int64_t code_base = cursor;
            if (head_has_int(h)) cursor += int64_t(keys) * values;
            const int64_t pivot_base = cursor;
            int pivot_index = 0;
            for (int k = 0; k < keys; ++k) {
                if (bits[h * keys + k] == 16) {
                    offsets_out[n++] = int32_t(pivot_base + 2 * int64_t(pivot_index) * values);
                    ++pivot_index;
                } else {
                    offsets_out[n++] = int32_t(code_base + k);
                }
            }
            cursor += 2 * int64_t(pivot_index) * values;
            strides[h] = code_base;
        }
    } else {
        for (int h = 0; h < heads; ++h) {
            int64_t local = 0;
            for (int k = 0; k < keys; ++k) {
                const int b = bits[h * keys + k];
                if (b == 16) local = (local + 1) / 2 * 2;
                offsets_out[n++] = int32_t(cursor + local);
                local += (tile * b + 7) / 8;  // 3/5 bits (extension): a KDA chunk rounds up to whole bytes
            }
            const int64_t stride = (local + 1) / 2 * 2;
            strides[h] = stride;
            cursor += stride * (values / tile);
        }
    }
    for (int h = 0; h < heads; ++h) offsets_out[n++] = int32_t(strides[h]);
    cursor = (cursor + 1) / 2 * 2;
    for (int h = 0; h < heads; ++h) {
        for (int k = 0; k < keys; ++k) {
            const int b = bits[h * keys + k];
            rows_out[h * keys + k] = b != 16 ? int32_t(cursor) : -1;
            if (b != 16) cursor += 2 * ((b == 2 && !kda) ? values / value_group_size : 1);
        }
    }
    for (int h = 0; h < heads; ++h) {
        const bool any = head_has_int(h);
        columns_out[h] = any ? int32_t(cursor) : -1;
        if (any) cursor += 2 * int64_t(values);
    }
    if (storage == 1) cursor = (cursor + 15) / 16 * 16;
    if (cursor > INT32_MAX) return SQ_ERR_SHAPE;
    *page_bytes_out = cursor;
    return SQ_OK;
}

int32_t sq_encode(const sq_plan *plan, const float *state, const int64_t *slots, int32_t batch, uint8_t *pages,
                  int64_t num_slots, int32_t *status, sq_stream_t stream) {
    if (int32_t e = check_plan(plan)) return e;
    if (batch < 0 || num_slots < 1) return SQ_ERR_ARGUMENT;
    if (batch == 0) return SQ_OK;
    if (!state || !slots || !pages) return SQ_ERR_ARGUMENT;
    sq::TileParams t = base_params(plan, pages, num_slots, slots, status);
    t.dense_in = state;
    return run(sq::kEncode, t, batch, stream);
}

int32_t sq_decode(const sq_plan *plan, const uint8_t *pages, int64_t num_slots, const int64_t *slots,
                  int32_t batch, float *state, int32_t *status, sq_stream_t stream) {
    if (int32_t e = check_plan(plan)) return e;
    if (batch < 0 || num_slots < 1) return SQ_ERR_ARGUMENT;
    if (batch == 0) return SQ_OK;
    if (!state || !slots || !pages) return SQ_ERR_ARGUMENT;
    sq::TileParams t = base_params(plan, const_cast<uint8_t *>(pages), num_slots, slots, status);
    t.dense_out = state;
    return run(sq::kDecode, t, batch, stream);
}

int32_t sq_step(const sq_plan *plan, uint8_t *pages, int64_t num_slots, const int64_t *slots, int32_t batch,
                const sq_step_args *args, float *state_out, int32_t *status, sq_stream_t stream) {
    if (int32_t e = check_plan(plan)) return e;
    if (batch < 0 || num_slots < 1) return SQ_ERR_ARGUMENT;
    if (batch == 0) return SQ_OK;
    if (!slots || !pages) return SQ_ERR_ARGUMENT;
    if (int32_t e = check_step(plan, args)) return e;
    sq::TileParams t = base_params(plan, pages, num_slots, slots, status);
    t.step = *args;
    t.dense_out = state_out;
    return run(sq::kStep, t, batch, stream);
}

int64_t sq_scratch_floats(const sq_plan *plan) {
    if (check_plan(plan) != SQ_OK) return -1;
    return int64_t(plan->heads) * (plan->values + 2 * plan->keys);
}

int32_t sq_readout(const sq_plan *plan, uint8_t *pages, int64_t num_slots, const int64_t *slots, int32_t batch,
                   const sq_step_args *args, float *scratch, int64_t *stable_slots, int32_t *status,
                   sq_stream_t stream) {
    if (int32_t e = check_plan(plan)) return e;
    if (batch < 0 || num_slots < 1) return SQ_ERR_ARGUMENT;
    if (batch == 0) return SQ_OK;
    if (!slots || !pages || !scratch || !stable_slots) return SQ_ERR_ARGUMENT;
    if (int32_t e = check_step(plan, args)) return e;
    sq::TileParams t = base_params(plan, pages, num_slots, slots, status);
    t.step = *args;
    t.scratch = scratch;
    t.stable_slots = stable_slots;
    t.scratch_stride = sq_scratch_floats(plan);
    return run(sq::kReadout, t, batch, stream);
}

int32_t sq_writeback(const sq_plan *plan, uint8_t *pages, int64_t num_slots, const int64_t *stable_slots,
                     int32_t batch, const float *scratch, float *state_out, int32_t *status, sq_stream_t stream) {
    if (int32_t e = check_plan(plan)) return e;
    if (batch < 0 || num_slots < 1) return SQ_ERR_ARGUMENT;
    if (batch == 0) return SQ_OK;
    if (!stable_slots || !pages || !scratch || state_out) return SQ_ERR_ARGUMENT;  // state_out is reserved
    sq::TileParams t = base_params(plan, pages, num_slots, stable_slots, status);
    t.scratch = const_cast<float *>(scratch);
    t.scratch_stride = sq_scratch_floats(plan);
    return run(sq::kWriteback, t, batch, stream);
}

int32_t sq_fit_state(const sq_plan *plan, const float *x, int32_t batch, int16_t *z, uint16_t *r, uint16_t *c,
                     uint16_t *r2, float *recon, sq_stream_t stream) {
    if (int32_t e = check_plan(plan)) return e;
    if (batch < 0) return SQ_ERR_ARGUMENT;
    if (batch == 0) return SQ_OK;
    if (!x || !z || !r || !c) return SQ_ERR_ARGUMENT;
    sq::TileParams t = base_params(plan, nullptr, 1, nullptr, nullptr);
    t.dense_in = x;
    t.fit_z = z;
    t.fit_r = r;
    t.fit_c = c;
    t.fit_r2 = r2;
    t.fit_recon = recon;
    return cuda_status(sq::launch_tile(sq::kFit, t, batch * plan->heads, stream));
}

int32_t sq_pack(const int16_t *codes, int64_t n, int32_t bits, uint8_t *out, sq_stream_t stream) {
    if (bits < 2 || bits > 8 || bits == 7) return SQ_ERR_ARGUMENT;
    if (n < 0 || (n > 0 && (!codes || !out))) return SQ_ERR_ARGUMENT;
    return cuda_status(sq::launch_pack(codes, n, bits, out, stream));
}

int64_t sq_packed_bytes(int64_t n, int32_t bits) {
    if (bits < 2 || bits > 8 || bits == 7) return -1;
    if (n < 0) return -1;
    return sq::packed_bytes(n, bits);
}

int32_t sq_unpack(const uint8_t *data, int64_t count, int32_t bits, int16_t *out, sq_stream_t stream) {
    if (bits < 2 || bits > 8 || bits == 7) return SQ_ERR_ARGUMENT;
    if (count < 0 || (count > 0 && (!data || !out))) return SQ_ERR_ARGUMENT;
    return cuda_status(sq::launch_unpack(data, count, bits, out, stream));
}

int32_t sq_fp32_step(float *state, int64_t num_slots, int32_t heads, int32_t keys, int32_t values, int32_t kda,
                     const int64_t *slots, int32_t batch, const sq_step_args *args, int32_t *status,
                     sq_stream_t stream) {
    if (batch < 0 || num_slots < 1 || heads < 1) return SQ_ERR_ARGUMENT;
    if (!pow2_dim(keys) || !pow2_dim(values)) return SQ_ERR_SHAPE;
    if (batch == 0) return SQ_OK;
    if (!state || !slots) return SQ_ERR_ARGUMENT;
    sq_plan p{};
    p.heads = heads;
    if (int32_t e = check_step(&p, args)) return e;
    return cuda_status(sq::launch_fp32_step(state, num_slots, heads, keys, values, kda, slots, batch, *args, status,
                                            stream));
}

int32_t sq_selftest_fp16_division(const float *a, const uint16_t *b, float *out, int64_t n, sq_stream_t stream) {
    if (n < 0 || (n > 0 && (!a || !b || !out))) return SQ_ERR_ARGUMENT;
    return cuda_status(sq::launch_division_selftest(a, b, out, n, stream));
}

}  // extern "C"
