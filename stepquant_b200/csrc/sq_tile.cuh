// Internal launch interface of the tile kernels (not part of the C ABI).
#pragma once

#include <cuda_runtime.h>

#include "sq_common.cuh"

namespace sq {

enum Mode { kEncode = 0, kDecode = 1, kStep = 2, kReadout = 3, kWriteback = 4, kFit = 5 };

struct TileParams {
    sq_plan plan;
    uint8_t *pages;
    int64_t num_slots;
    const int64_t *slots;  // request slots (stable slots for kWriteback)
    sq_step_args step;
    const float *dense_in;    // kEncode / kFit input
    float *dense_out;         // kDecode output, or the pre-quantization state of kStep / kWriteback
    float *scratch;           // kReadout writes, kWriteback reads
    int64_t *stable_slots;    // kReadout writes
    int64_t scratch_stride;   // floats per request
    int16_t *fit_z;
    uint16_t *fit_r;
    uint16_t *fit_c;
    uint16_t *fit_r2;
    float *fit_recon;
    int32_t *status;
    int skip_fast;  // tile kernel: leave heads that fast_head() accepts to the fast kernel
    int skip_pivot;  // tile kernel: leave GDN fp16 pivot heads to the pivot kernel
    int skip_two;    // tile kernel: leave GDN 2-bit heads to the 2-bit kernel
    int stage_inputs;  // fast kernels: q/k/v (or writeback scratch) rows are 16-byte aligned -> cp.async staging
    int stage_gates;   // fast kernels: fp32 gates -> cp.async staging
};

size_t tile_smem_bytes(int K, int V, int groups);
cudaError_t launch_tile(int mode, const TileParams &p, int items, cudaStream_t stream);

// Register-resident kernels for K = V = 128 GDN heads of width 4, 6 or 8
// (sq_fast.cu) for the step, readout, writeback, encode and decode modes.
// fast_eligible(): the plan's shape and the page alignment allow them;
// fast_head(): a head of that width is handled by them.  launch_fast also
// runs the fp16 pivot heads that pivot_heads() lists (a second kernel; none
// in the writeback, whose pivot values the readout already wrote) and the
// 2-bit heads that two_heads() lists.  The tile kernel handles the other heads
// (pivot or 2-bit heads when the plan has no host copy of its bits or more than
// 32 of them; 2-bit heads with value groups other than 32).
bool fast_eligible(const sq_plan &plan, const void *pages);
__host__ __device__ inline bool fast_head(const sq_plan &plan, int width) {
    return plan.architecture == SQ_GDN && plan.keys == 128 && plan.values == 128 &&
           (width == 4 || width == 6 || width == 8);
}
constexpr int kMaxPivotHeads = 32;
struct PivotHeads {
    int count;
    int ids[kMaxPivotHeads];
};
bool pivot_heads(const sq_plan &plan, PivotHeads *out);
cudaError_t launch_fast(int mode, const TileParams &p, int batch, cudaStream_t stream);

// GDN 2-bit heads (value groups of 32, K = V = 128) on their own kernel
// (sq_fast_two.cu), one CTA per (request, head), every mode; launch_fast runs
// it for the heads that two_heads() lists (none without a host copy of the
// bits or with more than kMaxTwoHeads of them: the tile kernel takes them).
constexpr int kMaxTwoHeads = 32;
struct TwoHeads {
    int count;
    int ids[kMaxTwoHeads];
};
bool two_heads(const sq_plan &plan, TwoHeads *out);
cudaError_t launch_two(int mode, const TileParams &p, const TwoHeads &th, int batch, cudaStream_t stream);

// Register-resident kernels for KDA heads with K = V = 128 (sq_fast_kda.cu):
// a head qualifies when it has integer rows and its code region (stride x
// V / 4 value tiles) fits the kernel's stage buffer.
constexpr int kKdaCodeCap = 12288;
__host__ __device__ inline bool kda_head_fits(int64_t stride, int values, int columns_offset) {
    return columns_offset >= 0 && stride * (values / 4) <= kKdaCodeCap;
}
bool kda_fast_eligible(const sq_plan &plan);
cudaError_t launch_fast_kda(int mode, const TileParams &p, int batch, cudaStream_t stream);

// Device-side: is `head` handled by a register-resident kernel (so the tile
// kernel, launched with skip_fast, leaves it)?
__device__ inline bool fast_head_dev(const sq_plan &P, int head) {
    if (P.storage != 0) return false;
    if (P.architecture == SQ_GDN) return fast_head(P, P.bits[head * P.keys]);  // (pivot heads: skip_pivot)
    return P.keys == 128 && P.values == 128 &&
           kda_head_fits(P.offsets[P.heads * P.keys + head], P.values, P.columns[head]);
}

}  // namespace sq
